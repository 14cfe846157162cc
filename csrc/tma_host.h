// Host-side construction of TMA tensor maps.  The driver entry point is looked
// up at run time through the CUDA runtime, so the extension does not link
// against libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace dmad {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || p == nullptr || q != cudaDriverEntryPointSuccess)
      throw std::runtime_error("dmad: cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// The encode call is a driver API function and needs a current context.  A host thread that has made
// no runtime call yet (the autograd engine's device thread running a backward, for instance) has
// none: cudaSetDevice on the current device makes its primary context current (it allocates nothing),
// once per thread.
inline void ensure_context() {
  static thread_local bool done = false;
  if (!done) {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
    done = true;
  }
}

// bf16 tensor map with a 128-byte swizzle.  dims/strides are innermost-first;
// strides are in bytes for dims 1..rank-1 (dim 0 is contiguous).  Every
// stride must be a multiple of 16 bytes and the base 16-byte aligned.
inline CUtensorMap make_tmap_bf16(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                                  const uint32_t* box, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("dmad: TMA base not 16B aligned");
  ensure_context();
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    s[i] = strides_bytes[i];
    if (s[i] % 16 != 0) throw std::runtime_error("dmad: TMA stride not a multiple of 16 bytes");
  }
  CUresult r = get_encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, es,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("dmad: cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return m;
}

}  // namespace dmad
