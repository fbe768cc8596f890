// Operand preparation kernels for the tensor-core path (HBM-bound, no GEMM shape).
//
//  * round_tf32_rne: TF32 round-to-nearest-even of an FP32 word, keeping
//    infinities and NaNs (the rule of the reference's round_tf32_even,
//    src/matmul_custom.cuh:158-164, and of src/precision.py:66-76).  The
//    tensor core ignores the 13 low fraction bits of a TF32 operand, so inputs
//    are rounded here first.
//  * pack_rows: copy a rows x cols row-major matrix with arbitrary (element)
//    alignment into a 16-byte aligned rows x ld_dst buffer, zero-filling the
//    padding columns, optionally TF32-rounding.  Used when an operand cannot be
//    described by a TMA tensor map (base not 16-byte aligned, or a row pitch
//    that is not a multiple of 16 bytes) and for every TF32 operand.
//  * round_tf32_vec: the aligned TF32 case as a float4 streaming kernel.
//  * convert_f32: FP32 -> BF16/FP16 (round to nearest even) or TF32-rounded FP32,
//    the device-side replacement of the harness's `.to(dtype)` after H2D.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

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

template <typename T, bool ROUND_TF32>
__global__ void pack_rows_kernel(const T *__restrict__ src, T *__restrict__ dst, int64_t rows, int64_t cols,
                                 int64_t ld_dst)
{
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const T *s = src + r * cols;
        T *d = dst + r * ld_dst;
        for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < ld_dst;
             col += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            T v;
            if (col < cols) {
                v = s[col];
                if constexpr (ROUND_TF32)
                    v = round_tf32_rne(v);
            } else {
                v = T(0.0f);
            }
            d[col] = v;
        }
    }
}

__global__ void round_tf32_vec_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, int64_t count4)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 v = src[i];
        v.x = round_tf32_rne(v.x);
        v.y = round_tf32_rne(v.y);
        v.z = round_tf32_rne(v.z);
        v.w = round_tf32_rne(v.w);
        dst[i] = v;
    }
}

// dst (n x ld_dst, K-major) = TF32-rounded transpose of src (k x n, row-major),
// zero in the padding columns k .. ld_dst-1.  32 x 32 tiles through shared
// memory so that both the global reads (along n) and writes (along k) coalesce.
// The tensor core reads MN-major TF32 operands only in a 32-byte-atom swizzle,
// so the TF32 path hands it a K-major B produced here, in the same pass that
// rounds the values.
__global__ void transpose_round_tf32_kernel(const float *__restrict__ src, float *__restrict__ dst, int64_t k,
                                            int64_t n, int64_t ld_dst)
{
    __shared__ float tile[32][33];
    const int64_t n_tiles = (n + 31) / 32;
    const int64_t k_tiles = (ld_dst + 31) / 32;
    for (int64_t kt = blockIdx.y; kt < k_tiles; kt += gridDim.y) {
        for (int64_t nt = blockIdx.x; nt < n_tiles; nt += gridDim.x) {
            const int64_t n0 = nt * 32, k0 = kt * 32;
            for (int r = threadIdx.y; r < 32; r += blockDim.y) {
                const int64_t kk = k0 + r, nn = n0 + threadIdx.x;
                tile[r][threadIdx.x] = (kk < k && nn < n) ? round_tf32_rne(src[kk * n + nn]) : 0.0f;
            }
            __syncthreads();
            for (int r = threadIdx.y; r < 32; r += blockDim.y) {
                const int64_t nn = n0 + r, kk = k0 + threadIdx.x;
                if (nn < n && kk < ld_dst)
                    dst[nn * ld_dst + kk] = tile[threadIdx.x][r];
            }
            __syncthreads();
        }
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
