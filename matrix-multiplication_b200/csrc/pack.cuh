// Operand preparation kernels for the tensor-core path (HBM-bound, no GEMM shape).
//
//  * round_tf32_rne: TF32 round-to-nearest-even of an FP32 word, keeping
//    infinities and NaNs (the rule of the reference's round_tf32_even,
//    src/matmul_custom.cuh:158-164, and of src/precision.py:66-76), for the
//    conversion kernel, the FFMA kernel's small-TF32 form and the FP64 check.
//  * pack_pair: copy rows x cols row-major operands with arbitrary (element)
//    alignment into 16-byte aligned rows x ld buffers, zero-filling the padding
//    columns -- A and B in one launch.  Used when an operand cannot be described
//    by a TMA tensor map (base not 16-byte aligned, or a row pitch that is not a
//    multiple of 16 bytes); TF32 operands are copied unrounded, the TMA loads of
//    their TFLOAT32 tensor maps round them.
//  * convert_f32: FP32 -> BF16/FP16 (round to nearest even) or TF32-rounded FP32,
//    the device-side replacement of the harness's `.to(dtype)` after H2D.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"

namespace b200 {

__device__ __forceinline__ uint32_t round_tf32_rne_bits(uint32_t bits)
{
    if ((bits & 0x7f800000u) != 0x7f800000u)
        bits = (bits + 0xfffu + ((bits >> 13) & 1u)) & 0xffffe000u;
    return bits;
}

__device__ __forceinline__ float round_tf32_rne(float x)
{
    return __uint_as_float(round_tf32_rne_bits(__float_as_uint(x)));
}

// One repack job: rows x cols (row-major, element-aligned) -> rows x ld, zero in
// columns cols..ld-1.  rows == 0 means the operand needs no copy.
template <typename T>
struct PackJob {
    const T *src;
    T *dst;
    int64_t rows, cols, ld;
};

// Both FP16/BF16 operands that TMA cannot read in place, in one launch: blocks
// [0, a_blocks) copy job a, the rest job b, each a grid-stride loop over the
// destination's elements (coalesced on both sides).
template <typename T>
__global__ void __launch_bounds__(256) pack_pair_kernel(const PackJob<T> a, const PackJob<T> b, int a_blocks)
{
    wait_for_prior_grid();
    allow_next_grid();
    const bool first = static_cast<int>(blockIdx.x) < a_blocks;
    const PackJob<T> job = first ? a : b;
    const int64_t blocks = first ? a_blocks : static_cast<int64_t>(gridDim.x) - a_blocks;
    const int64_t block = first ? blockIdx.x : blockIdx.x - a_blocks;
    const int64_t total = job.rows * job.ld;
    for (int64_t i = block * 256 + threadIdx.x; i < total; i += blocks * 256) {
        const int64_t r = i / job.ld, col = i % job.ld;
        job.dst[i] = col < job.cols ? job.src[r * job.cols + col] : T(0.0f);
    }
}

template <typename T>
__device__ __forceinline__ T convert_one(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 convert_one<__nv_bfloat16>(float x)
{
    return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half convert_one<__half>(float x)
{
    return __float2half_rn(x);
}
template <>
__device__ __forceinline__ float convert_one<float>(float x)
{
    return round_tf32_rne(x);
}

template <typename T>
__global__ void convert_f32_kernel(const float *__restrict__ src, T *__restrict__ dst, int64_t count)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = convert_one<T>(src[i]);
}

} // namespace b200
