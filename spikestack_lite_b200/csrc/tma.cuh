// Tensor-memory-accelerator helpers shared by the tcgen05 kernels: the 2-D
// tiled load into this CTA's own shared memory and host-side encoding of fp32
// row-major tensor maps through the driver entry point.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "spk_common.cuh"

namespace spk {

// One box of a 2-D tensor map into shared memory, completing `bar`'s
// transaction count.  x = column (innermost) coordinate, y = row.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst_smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// fp32 row-major [rows, cols] with a row pitch of `pitch` elements, boxes of
// box_cols x box_rows, zero fill outside the tensor.  `what` names the tensor
// in the error message.
inline int make_map_2d_f32(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t pitch,
                           int box_cols, int box_rows, const char* what) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(SPK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch * 4) % 16 != 0)
    return fail(SPK_EINVAL, "%s: base must be 16-byte aligned and the row pitch a multiple of 16 bytes", what);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SPK_ECUDA, "cuTensorMapEncodeTiled failed (%d) for %s [%lld, %lld]", (int)r, what, (long long)rows,
                (long long)cols);
  return SPK_OK;
}

// 32-bit words [rows, cols] (packed spikes: bit b of word w = column 32w + b)
// with a row pitch of `pitch` words, boxes of box_cols x box_rows words, no
// swizzle, zero fill outside the tensor.  box_cols * 4 must be a multiple of 16.
inline int make_map_2d_u32(CUtensorMap* map, const uint32_t* base, int64_t rows, int64_t cols, int64_t pitch,
                           int box_cols, int box_rows, const char* what) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(SPK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch * 4) % 16 != 0 || (box_cols * 4) % 16 != 0)
    return fail(SPK_EINVAL, "%s: base 16-byte aligned, row pitch and box width multiples of 16 bytes", what);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch * sizeof(uint32_t)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SPK_ECUDA, "cuTensorMapEncodeTiled failed (%d) for %s [%lld, %lld]", (int)r, what, (long long)rows,
                (long long)cols);
  return SPK_OK;
}

// Four packed spikes (the low 4 bits of `nib`) as the fp32 bit patterns of
// 1.0f / 0.0f: exactly what a load of the unpacked fp32 spikes would give.
__device__ __forceinline__ uint4 nibble_f32x4(uint32_t nib) {
  return make_uint4((nib & 1u) ? 0x3f800000u : 0u, (nib & 2u) ? 0x3f800000u : 0u, (nib & 4u) ? 0x3f800000u : 0u,
                    (nib & 8u) ? 0x3f800000u : 0u);
}

// As make_map_2d_f32 with the 128-byte swizzle: box_cols * 4 must be 128, and
// each box lands as 128-byte rows in 1024-byte atoms with the 16-byte chunks
// of row r XOR-permuted by r & 7 -- the K-major UMMA operand layout.
inline int make_map_2d_swizzled_f32(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t pitch,
                                    int box_cols, int box_rows, const char* what) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(SPK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch * 4) % 16 != 0 || box_cols * 4 != 128)
    return fail(SPK_EINVAL, "%s: base 16-byte aligned, row pitch a multiple of 16 bytes, 32-column boxes", what);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SPK_ECUDA, "cuTensorMapEncodeTiled (swizzled) failed (%d) for %s [%lld, %lld]", (int)r, what,
                (long long)rows, (long long)cols);
  return SPK_OK;
}

}  // namespace spk
