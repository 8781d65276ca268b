// tc_host.h — host helpers for the tcgen05 kernels: TMA tensor maps and the SM count.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

namespace sjb {
namespace tc {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D bf16 row-major tensor [rows, inner] with `row_bytes` pitch; box of
// box_rows x box_inner elements, 128-byte swizzle (box_inner * 2 == 128).
// The base address and pitch must be 16-byte aligned.
inline bool make_map_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                          uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2D tensor of bytes (fp8 e4m3 codes) [rows, inner], box of box_rows x 128
// bytes, 128-byte swizzle: the same shared-memory layout as a bf16 box of 64.
inline bool make_map_u8(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2D fp32 row-major tensor, box of box_rows x box_inner (box_inner * 4 == 128), 128-byte swizzle.
inline bool make_map_f32(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                         uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// Raise a kernel's dynamic shared-memory limit to `bytes` on the current
// device.  The attribute belongs to the device, so it is set once per device
// ordinal (bit d of `done`); ordinals >= 64 set it on every call.  Safe from
// several host threads: two threads that race both set the same value.
template <typename Kernel>
inline cudaError_t ensure_smem_attr(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess) return rc;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  rc = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (rc == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return rc;
}

}  // namespace tc
}  // namespace sjb
