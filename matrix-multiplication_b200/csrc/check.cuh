// FP64 verification of a GEMM output on the GPU (matmul_check_fp64).
//
// The reference validates every output against an FP64 product of the
// precision-rounded inputs with a roundoff-aware allowance (src/precision.py:
// GemmReference, :99-161):  |C - ref| <= atol + rtol |ref| + gamma_K (|A| |B|),
// atol = rtol = 5e-4, gamma_K from u = 2^-23.  On the CPU that is O(MKN) in FP64
// and takes minutes at 8192^3; this kernel computes the same per-output ratio
// |C - ref| / allowance for every output on the GPU and reduces its maximum
// (and the maximum |C - ref|).  For TF32 the magnitude term uses the upper
// envelope of the legal input models (RNE, ties-away and unrounded FP32), as the
// reference does.
//
// 64 x 64 outputs per 256-thread block (4 x 4 per thread), K in steps of 16
// through shared memory as doubles.  A non-finite output gives an infinite ratio.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "pack.cuh"

namespace b200 {

constexpr int CK_TILE = 64;
constexpr int CK_BK = 16;

__device__ unsigned long long g_check_result[2];   // max ratio, max |C - ref| (double bits)

template <typename T>
__device__ __forceinline__ void check_operand(T x, double &value, double &magnitude);

template <>
__device__ __forceinline__ void check_operand<__nv_bfloat16>(__nv_bfloat16 x, double &value, double &magnitude)
{
    value = static_cast<double>(__bfloat162float(x));
    magnitude = fabs(value);
}

template <>
__device__ __forceinline__ void check_operand<__half>(__half x, double &value, double &magnitude)
{
    value = static_cast<double>(__half2float(x));
    magnitude = fabs(value);
}

// FP32 storage: pedantic FP32 (TF32 = false) or TF32 (RNE model, envelope magnitude).
template <bool TF32>
__device__ __forceinline__ void check_float(float x, double &value, double &magnitude)
{
    if constexpr (TF32) {
        const uint32_t bits = __float_as_uint(x);
        const float rne = round_tf32_rne(x);
        const uint32_t away_bits =
            (bits & 0x7f800000u) == 0x7f800000u ? bits : ((bits + 0x1000u) & 0xffffe000u);
        value = static_cast<double>(rne);
        magnitude = fmax(fmax(fabs(value), fabs(static_cast<double>(__uint_as_float(away_bits)))),
                         fabs(static_cast<double>(x)));
    } else {
        value = static_cast<double>(x);
        magnitude = fabs(value);
    }
}

template <typename T, bool TF32>
__global__ void __launch_bounds__(256)
fp64_check_kernel(const T *__restrict__ a, const T *__restrict__ b, const float *__restrict__ c, int m, int n,
                  int k, double gamma)
{
    __shared__ double av[CK_BK][CK_TILE], am[CK_BK][CK_TILE];
    __shared__ double bv[CK_BK][CK_TILE], bm[CK_BK][CK_TILE];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    double worst_ratio = 0.0, worst_diff = 0.0;
    for (int64_t tile = blockIdx.x; tile < static_cast<int64_t>((m + CK_TILE - 1) / CK_TILE) *
                                               ((n + CK_TILE - 1) / CK_TILE);
         tile += gridDim.x) {
        const int tiles_n = (n + CK_TILE - 1) / CK_TILE;
        const int m0 = static_cast<int>(tile / tiles_n) * CK_TILE;
        const int n0 = static_cast<int>(tile % tiles_n) * CK_TILE;
        double ref[4][4] = {}, mag[4][4] = {};
        for (int k0 = 0; k0 < k; k0 += CK_BK) {
            for (int i = threadIdx.x; i < CK_BK * CK_TILE; i += 256) {
                const int kk = i / CK_TILE, r = i % CK_TILE;   // A: row m0 + r, column k0 + kk
                double v = 0.0, g = 0.0;
                if (m0 + r < m && k0 + kk < k) {
                    if constexpr (sizeof(T) == 4)
                        check_float<TF32>(a[static_cast<size_t>(m0 + r) * k + k0 + kk], v, g);
                    else
                        check_operand<T>(a[static_cast<size_t>(m0 + r) * k + k0 + kk], v, g);
                }
                av[kk][r] = v;
                am[kk][r] = g;
                v = g = 0.0;                                     // B: row k0 + kk, column n0 + r
                if (k0 + kk < k && n0 + r < n) {
                    if constexpr (sizeof(T) == 4)
                        check_float<TF32>(b[static_cast<size_t>(k0 + kk) * n + n0 + r], v, g);
                    else
                        check_operand<T>(b[static_cast<size_t>(k0 + kk) * n + n0 + r], v, g);
                }
                bv[kk][r] = v;
                bm[kk][r] = g;
            }
            __syncthreads();
#pragma unroll 4
            for (int kk = 0; kk < CK_BK; ++kk) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const double x = av[kk][ty + 16 * i], xm = am[kk][ty + 16 * i];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        ref[i][j] = fma(x, bv[kk][tx + 16 * j], ref[i][j]);
                        mag[i][j] = fma(xm, bm[kk][tx + 16 * j], mag[i][j]);
                    }
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = m0 + ty + 16 * i;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = n0 + tx + 16 * j;
                if (row < m && col < n) {
                    const double got = static_cast<double>(c[static_cast<size_t>(row) * n + col]);
                    const double diff = fabs(got - ref[i][j]);
                    const double allow = 5e-4 + 5e-4 * fabs(ref[i][j]) + gamma * mag[i][j];
                    double ratio = diff / allow;
                    if (!isfinite(got) || isnan(ratio))
                        ratio = __longlong_as_double(0x7ff0000000000000ll);
                    worst_ratio = fmax(worst_ratio, ratio);
                    worst_diff = isfinite(diff) ? fmax(worst_diff, diff) : worst_diff;
                }
            }
        }
    }
    // Non-negative doubles order like their bit patterns.
    for (int off = 16; off; off >>= 1) {
        worst_ratio = fmax(worst_ratio, __shfl_xor_sync(0xffffffffu, worst_ratio, off));
        worst_diff = fmax(worst_diff, __shfl_xor_sync(0xffffffffu, worst_diff, off));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&g_check_result[0], static_cast<unsigned long long>(__double_as_longlong(worst_ratio)));
        atomicMax(&g_check_result[1], static_cast<unsigned long long>(__double_as_longlong(worst_diff)));
    }
}

} // namespace b200
