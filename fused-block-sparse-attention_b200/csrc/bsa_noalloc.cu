// bsa_sel_csr_noalloc: the CSR transpose of a selection without any device
// allocation by the caller or by the library.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) at the
// point where they build the transpose — code running while a memory pool is
// locked or exhausted, embedders whose host language owns every device
// allocation through its own arena and forbids side allocations, and real-time
// loops that must not enter the driver's allocator.  They still pass the
// selection and the row_ptr / col outputs; the temporary storage (per-key-block
// counts, radix-sort keys and values, the sort/scan scratch) lives in one
// file-scope device array of kNoAllocScratchBytes that every GPU loading this
// library holds until the process exits.
//
// Rules of use:
//  - The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.  The address is cached for the life of the
//    process: it does not survive cudaDeviceReset of that device.
//  - All calls on a device share the array, which keeps the previous call's
//    contents; the counts that must start at zero are cleared by every call.
//    Calls whose work overlaps on the GPU (different streams, or different host
//    threads without ordering) race on the array and corrupt each other.
//  - Selections whose scratch need exceeds kNoAllocScratchBytes are rejected
//    with BSA_ERR_UNSUPPORTED (about one million (query block, slot) entries).
#include <mutex>
#include <string>

#include "bsa_host.h"

namespace bsa {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB

static __device__ __align__(256) unsigned char g_csr_scratch[kNoAllocScratchBytes];

// Device address of g_csr_scratch per device (the host-side name is only a
// stand-in and must never be handed to a kernel).
static constexpr int kMaxDevices = 64;
static void *g_scratch_ptr[kMaxDevices];
static std::mutex g_scratch_mu;

static bsa_status scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(BSA_ERR_LAUNCH, std::string("sel_csr_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(BSA_ERR_UNSUPPORTED, "sel_csr_noalloc: device index too large");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_csr_scratch);
    if (e != cudaSuccess || !p)
      return fail(BSA_ERR_LAUNCH, std::string("sel_csr_noalloc: cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BSA_OK;
}

}  // namespace bsa

extern "C" bsa_status bsa_sel_csr_noalloc(const bsa_csr_args *a, bsa_stream_t stream) {
  using namespace bsa;
  const size_t need = bsa_csr_workspace(a);
  if (need == 0) return bsa_sel_csr(a, nullptr, 0, stream);  // reports the argument error
  if (need > kNoAllocScratchBytes)
    return fail(BSA_ERR_UNSUPPORTED, "sel_csr_noalloc: selection needs " + std::to_string(need) +
                                         " bytes of scratch, more than the fixed " +
                                         std::to_string(kNoAllocScratchBytes) +
                                         "; use bsa_sel_csr with a caller workspace");
  void *ws = nullptr;
  if (bsa_status s = scratch_address(&ws)) return s;
  return bsa_sel_csr(a, ws, kNoAllocScratchBytes, stream);
}
