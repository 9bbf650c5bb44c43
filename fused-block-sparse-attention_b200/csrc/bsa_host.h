// Host-side helpers shared by the launchers: error reporting and TMA
// tensor-map encoding.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/bsa.h"

namespace bsa {

// Records a thread-local error message and returns `st`.
bsa_status fail(bsa_status st, const std::string &msg);

// Maps the last CUDA runtime error (if any) to BSA_ERR_LAUNCH.
bsa_status check_launch(const char *what);

inline size_t elem_size(int dtype) { return dtype == BSA_F32 ? 4 : 2; }

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Encodes a 4-D tiled tensor map over a (B, H, L, D) view of 16-bit elements
// with a box of 64 columns x `rows` rows and 128-byte swizzle.  The three
// outer axes are ordered by increasing stride before encoding; `perm[i]` gives
// the encoded position (1..3) of axis i (0 = L, 1 = H, 2 = B).
struct TensorMap4 {
  CUtensorMap map;
  int perm[3];
};
bsa_status make_tmap(TensorMap4 *out, const void *ptr, int dtype, int B, int H, int L, int D,
                     int64_t sb, int64_t sh, int64_t sl, int rows, const char *name);

// Encodes a 3-D tiled tensor map over a contiguous fp32 (G, rows, dim) array
// with a box of 32 columns (128 bytes) x `box_rows` rows x 1 and 128-byte
// swizzle; rows past `rows` read as zero.  dim must be a multiple of 4.
bsa_status make_tmap_f32_rows(CUtensorMap *out, const float *ptr, int G, int rows, int dim,
                              int box_rows, const char *name);

}  // namespace bsa
