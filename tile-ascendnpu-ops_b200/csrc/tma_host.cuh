// Host-side TMA tensor maps.
//
// cuTensorMapEncodeTiled is a driver API call; the library reaches it through
// the runtime's driver entry point, so it links no libcuda import.  Every map
// built here uses the 128-byte swizzle that the kernels' shared-memory tile
// addressing assumes (16-byte unit u of 128-byte row r at unit u ^ (r % 8)),
// zero fill for out-of-range boxes, and 256-byte L2 promotion.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace tileops {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// A tiled map of `rank` dims over 16-bit elements.  dims[0] is the innermost
// (contiguous) extent in elements; strides_bytes[i] is the byte stride of
// dims[i + 1].  box[0] * 2 must be 128 (one swizzle row).
inline bool make_tiled_map_16bit(CUtensorMap* map, const void* base, bool bf16, int rank,
                                 const uint64_t* dims, const uint64_t* strides_bytes,
                                 const uint32_t* box) {
  auto fn = tensor_map_encoder();
  if (!fn || rank < 1 || rank > 5) return false;
  cuuint64_t sizes[5];
  cuuint64_t strides[4];
  cuuint32_t boxes[5];
  cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    sizes[i] = dims[i];
    boxes[i] = box[i];
    if (i + 1 < rank) strides[i] = strides_bytes[i];
  }
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  rank, const_cast<void*>(base), sizes, strides, boxes, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D map over a (B, S, H, D) row-major tensor: dims (D, H, S, B), box
// (64, 1, rows, 1).
inline bool make_bshd_map(CUtensorMap* map, const void* base, int dim, int heads, int seq,
                          int batch, int rows, bool bf16) {
  const uint64_t dims[4] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(heads),
                            static_cast<uint64_t>(seq), static_cast<uint64_t>(batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(dim) * 2,
                               static_cast<uint64_t>(dim) * heads * 2,
                               static_cast<uint64_t>(dim) * heads * seq * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(rows), 1};
  return make_tiled_map_16bit(map, base, bf16, 4, dims, strides, box);
}

}  // namespace tileops
