// Host helpers: thread-local error text, CUDA error mapping and TMA tensor-map
// encoding through the driver entry point (no link-time libcuda dependency).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "bsa_host.h"

namespace bsa {

static thread_local std::string g_last_error;

bsa_status fail(bsa_status st, const std::string &msg) {
  g_last_error = msg;
  return st;
}

bsa_status check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(BSA_ERR_LAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  return BSA_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bsa_status make_tmap(TensorMap4 *out, const void *ptr, int dtype, int B, int H, int L, int D,
                     int64_t sb, int64_t sh, int64_t sl, int rows, const char *name) {
  if (dtype != BSA_BF16 && dtype != BSA_F16)
    return fail(BSA_ERR_DTYPE, std::string(name) + ": TMA path needs bf16/f16");
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return fail(BSA_ERR_STRIDE, std::string(name) + ": base pointer not 16-byte aligned");
  auto enc = get_encode();
  if (!enc) return fail(BSA_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  // Axis extents/strides; an axis of extent 1 gets a harmless large stride so
  // the stride ordering below stays well defined.
  int64_t ext[3] = {L, H, B};
  int64_t str[3] = {sl, sh, sb};
  const int64_t big = (int64_t)1 << 36;
  for (int i = 0; i < 3; ++i) {
    if (ext[i] == 1) str[i] = big + i * 8;
    if (str[i] <= 0 || (str[i] * 2) % 16)
      return fail(BSA_ERR_STRIDE, std::string(name) + ": strides must be positive multiples of 8 elements");
  }
  int order[3] = {0, 1, 2};
  std::sort(order, order + 3, [&](int a, int b) { return str[a] < str[b]; });
  cuuint64_t gdim[4];
  cuuint64_t gstride[3];
  cuuint32_t box[4];
  cuuint32_t estr[4] = {1, 1, 1, 1};
  gdim[0] = (cuuint64_t)D;
  box[0] = 64;
  for (int pos = 0; pos < 3; ++pos) {
    const int ax = order[pos];
    out->perm[ax] = pos + 1;
    gdim[pos + 1] = (cuuint64_t)ext[ax];
    gstride[pos] = (cuuint64_t)(str[ax] * 2);
    box[pos + 1] = (ax == 0) ? (cuuint32_t)rows : 1u;
  }
  CUresult r = enc(&out->map, dtype == BSA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void *>(ptr), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
    return fail(BSA_ERR_STRIDE, buf);
  }
  return BSA_OK;
}

bsa_status make_tmap_f32_rows(CUtensorMap *out, const float *ptr, int G, int rows, int dim,
                              int box_rows, const char *name) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 || dim % 4)
    return fail(BSA_ERR_STRIDE, std::string(name) + ": needs a 16-byte aligned base and dim % 4 == 0");
  auto enc = get_encode();
  if (!enc) return fail(BSA_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t gdim[3] = {(cuuint64_t)dim, (cuuint64_t)rows, (cuuint64_t)G};
  cuuint64_t gstride[2] = {(cuuint64_t)dim * 4, (cuuint64_t)dim * 4 * (cuuint64_t)rows};
  cuuint32_t box[3] = {32u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(ptr), gdim, gstride,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
    return fail(BSA_ERR_STRIDE, buf);
  }
  return BSA_OK;
}

}  // namespace bsa

extern "C" const char *bsa_last_error(void) { return bsa::g_last_error.c_str(); }
