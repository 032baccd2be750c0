// sdg_tma.h — host-side TMA tensor-map construction (fp16, 128-byte swizzle).
// The driver entry point is resolved through the runtime so the library does
// not link libcuda directly (it loads on machines without a GPU driver).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cstdint>

namespace sdg {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tensor with `rank` dims (dims[0] innermost, contiguous), byte strides for
// dims 1.., box extents; fp16 with 128B swizzle unless told otherwise.
// elem_strides (optional): traversal stride per dim (1 = every element; a box of extent e with
// stride s loads ceil(e / s) elements along that dim).
inline bool make_tmap(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
                      CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      const uint32_t* elem_strides = nullptr) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (elem_strides)
    for (int i = 0; i < rank && i < 5; ++i) estr[i] = elem_strides[i];
  CUresult r = enc(m, dtype, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Row-major [rows, cols] with row stride ld (elements); box = [box_rows, box_cols].
inline bool make_tmap_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows, uint32_t box_cols) {
  uint64_t dims[2] = {cols, rows};
  uint64_t str[1] = {ld * 2};
  uint32_t box[2] = {box_cols, box_rows};
  return make_tmap(m, base, 2, dims, str, box);
}

}  // namespace sdg
