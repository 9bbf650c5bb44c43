// Shared device primitives for the sm_100a kernels: mbarriers with bounded
// waits, TMA tile loads, ldmatrix, bf16/f16 mma.sync, 128B-swizzle addressing.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bsa.h"

namespace bsa {

// ---------------------------------------------------------------- status word
__device__ __forceinline__ void report(int32_t *status, int bit) {
  if (status) atomicOr(status, bit);
}

// ---------------------------------------------------------------- smem / mbar
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and the caller reports
// BSA_DEVERR_TIMEOUT) when the phase has not completed after kSpinLimit polls;
// each try_wait may itself suspend for a short hardware-defined interval.
constexpr uint32_t kSpinLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// The same bounded wait for a whole converged warp: the lanes poll together and
// a vote makes the outcome warp-uniform.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (__any_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return false;
}

// 4-D tiled TMA load (no multicast) of one box into shared memory, completing
// on `bar` with the box's byte count.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// TMA load addressed by (col, row, head, batch) on a map whose outer axes were
// reordered by stride: `perm` packs the encoded position (1..3) of the row,
// head and batch axes in bits [0:2), [2:4), [4:6).
__device__ __forceinline__ void tma_load_rhb(void *dst, const CUtensorMap *map, uint64_t *bar,
                                             int perm, int col, int row, int head, int batch) {
  const int pr = perm & 3, ph = (perm >> 2) & 3;
  const int c1 = pr == 1 ? row : (ph == 1 ? head : batch);
  const int c2 = pr == 2 ? row : (ph == 2 ? head : batch);
  const int c3 = pr == 3 ? row : (ph == 3 ? head : batch);
  tma_load_4d(dst, map, bar, col, c1, c2, c3);
}

// L2 prefetch of the same box tma_load_rhb would copy (no shared memory, no
// barrier): lets a producer run several ring stages ahead of its loads.
__device__ __forceinline__ void tma_prefetch_rhb(const CUtensorMap *map, int perm, int col, int row,
                                                 int head, int batch) {
  const int pr = perm & 3, ph = (perm >> 2) & 3;
  const int c1 = pr == 1 ? row : (ph == 1 ? head : batch);
  const int c2 = pr == 2 ? row : (ph == 2 ? head : batch);
  const int c3 = pr == 3 ? row : (ph == 3 ? head : batch);
  asm volatile(
      "cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(col), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- swizzle
// A tile of R rows x D cols (16-bit elements) is stored as D/64 regions of
// R x 128 bytes, each written by one TMA box with CU_TENSOR_MAP_SWIZZLE_128B:
// the 16-byte chunk c of row r sits at chunk c ^ (r & 7).  Region bases are
// 1024-byte aligned.
__device__ __forceinline__ uint32_t swz(uint32_t base, int R, int row, int col) {
  const int region = col >> 6;
  const int chunk = (col & 63) >> 3;
  return base + region * R * 128 + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// ---------------------------------------------------------------- ldmatrix / mma
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
struct Mma;

template <>
struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float *c, const uint32_t *a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

template <>
struct Mma<__half> {
  __device__ __forceinline__ static void run(float *c, const uint32_t *a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

// Barrier `id` (1..15) among `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Hardware base-2 exponential (the MUFU ex2 instruction, flush-to-zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// One rotary pair with transformers' op-by-op rounding to T (apply_rotary_pos_emb
// in the tensor dtype): y0 = x0*c0 + (-x1)*s0, y1 = x1*c1 + x0*s1, each product
// and each sum rounded to T.  Shared by bsa_rope, the rope-aware pooling and the
// in-kernel rotation of q so that all three produce identical values.
template <typename T>
__device__ __forceinline__ void rope_pair(T x0t, T x1t, T c0t, T s0t, T c1t, T s1t, T &y0, T &y1) {
  const float x0 = Mma<T>::to_f(x0t), x1 = Mma<T>::to_f(x1t);
  auto rd = [](float v) { return Mma<T>::to_f(Mma<T>::from_f(v)); };
  const float t0 = rd(__fmul_rn(x0, Mma<T>::to_f(c0t))), u0 = rd(__fmul_rn(-x1, Mma<T>::to_f(s0t)));
  const float t1 = rd(__fmul_rn(x1, Mma<T>::to_f(c1t))), u1 = rd(__fmul_rn(x0, Mma<T>::to_f(s1t)));
  y0 = Mma<T>::from_f(__fadd_rn(t0, u0));
  y1 = Mma<T>::from_f(__fadd_rn(t1, u1));
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes of
// work, each element rounded exactly as the scalar instruction would).
#define BSA_F32X2_OP(name, op)                                                            \
  __device__ __forceinline__ float2 name(float2 a, float2 b) {                             \
    float2 d;                                                                            \
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" \
        op " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                                  \
        : "=f"(d.x), "=f"(d.y)                                                           \
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));                                       \
    return d;                                                                            \
  }
BSA_F32X2_OP(add2, "add.rn.f32x2")
BSA_F32X2_OP(sub2, "sub.rn.f32x2")
BSA_F32X2_OP(mul2, "mul.rn.f32x2")
#undef BSA_F32X2_OP
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Three-input maximum (one sm_100 instruction; same result as two fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of 64 registers: 8 independent chains of three-input maxima.
__device__ __forceinline__ float max64(const float *s) {
  float m8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m8[i] = fmax3(s[i], s[i + 8], s[i + 16]);
#pragma unroll
  for (int c = 24; c < 56; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) m8[i] = fmax3(m8[i], s[c + i], s[c + 8 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m8[i] = fmaxf(m8[i], s[56 + i]);
  return fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
}

// ---------------------------------------------------------------- slot kinds
// Classification of one selected slot for one query block.
enum : int { KIND_SKIP = 0, KIND_FULL = 1, KIND_TRIU = 2, KIND_PAD = 4 };

// Kind of slot `slot` holding block id `kblk` for query block `qblk`.
// Duplicate detection (TOKEN mode) is done by the caller: pass dup = true when
// an earlier slot of the same row holds the same block id.
__device__ __forceinline__ int slot_kind(int kblk, int slot, bool dup, int qblk, int nblk, int bs,
                                         int L, int mask_mode, int causal, int32_t *status) {
  if (kblk < 0 || kblk >= nblk) {
    report(status, BSA_DEVERR_INDEX);
    return KIND_SKIP;
  }
  int k;
  if (mask_mode == BSA_MASK_SLOT) {
    if (!causal)
      k = KIND_FULL;
    else if (slot == 0)
      k = KIND_TRIU;
    else
      k = (kblk >= qblk) ? KIND_SKIP : KIND_FULL;
  } else {
    if (dup) return KIND_SKIP;
    if (causal) {
      if (kblk > qblk) return KIND_SKIP;
      k = (kblk == qblk) ? KIND_TRIU : KIND_FULL;
    } else {
      k = KIND_FULL;
    }
  }
  if (k != KIND_SKIP && (kblk + 1) * bs > L) k |= KIND_PAD;
  return k;
}

// Live-slot list of one selection row, built by a whole warp: lane l classifies
// slots l, l + 32, ... (slot_kind, with the TOKEN-mode duplicate test), and a
// ballot compacts the live ones in slot order, so put(pos, kblk, kind, slot) sees
// exactly the sequence a serial walk over the slots would produce.  selrow ==
// nullptr is the identity selection (slot j is key block j, kk = nblk).  At most
// maxn entries are kept; the return value (the same in every lane) is their
// count.  One global load per lane instead of kk dependent ones on one thread.
template <typename Put>
__device__ __forceinline__ int warp_live_slots(const int32_t *selrow, int kk, int maxn, int qblk,
                                               int nblk, int bs, int L, int mask_mode, int causal,
                                               int32_t *status, Put put) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int j0 = 0; j0 < kk && n < maxn; j0 += 32) {
    const int j = j0 + lane;
    int kb = 0, kind = KIND_SKIP;
    if (j < kk) {
      if (selrow) {
        kb = __ldg(selrow + j);
        bool dup = false;
        if (mask_mode == BSA_MASK_TOKEN)
          for (int i = 0; i < j && !dup; ++i) dup = __ldg(selrow + i) == kb;
        kind = slot_kind(kb, j, dup, qblk, nblk, bs, L, mask_mode, causal, status);
      } else {
        kb = j;
        kind = slot_kind(kb, kb, false, qblk, nblk, bs, L, mask_mode, causal, status);
      }
    }
    const unsigned live = __ballot_sync(0xffffffffu, kind != KIND_SKIP);
    const int pos = n + __popc(live & ((1u << lane) - 1u));
    if (kind != KIND_SKIP && pos < maxn) put(pos, kb, kind, j);
    n += __popc(live);
  }
  return n < maxn ? n : maxn;
}

// Largest kk for an explicit selection (slot table kept in shared memory).
constexpr int kMaxKK = 512;

// Fills s_slot[0..kk) with (kblk << 3) | kind for one selection row, using all
// threads of the block.  Must be followed by __syncthreads().
__device__ __forceinline__ void build_slot_table(int *s_slot, const int32_t *selrow, int kk,
                                                 int qblk, int nblk, int bs, int L, int mask_mode,
                                                 int causal, int32_t *status) {
  for (int j = threadIdx.x; j < kk; j += blockDim.x) {
    const int kb = __ldg(selrow + j);
    bool dup = false;
    if (mask_mode == BSA_MASK_TOKEN)
      for (int i = 0; i < j && !dup; ++i) dup = (__ldg(selrow + i) == kb);
    const int kind = slot_kind(kb, j, dup, qblk, nblk, bs, L, mask_mode, causal, status);
    s_slot[j] = kind == KIND_SKIP ? 0 : ((kb << 3) | kind);
  }
}

}  // namespace bsa
