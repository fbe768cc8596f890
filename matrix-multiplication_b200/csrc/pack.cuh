// Operand preparation kernels for the tensor-core path (HBM-bound, no GEMM shape).
//
//  * round_tf32_rne: TF32 round-to-nearest-even of an FP32 word, keeping
//    infinities and NaNs (the rule of the reference's round_tf32_even,
//    src/matmul_custom.cuh:158-164, and of src/precision.py:66-76).  The
//    tensor core ignores the 13 low fraction bits of a TF32 operand, so inputs
//    are rounded here first.
//  * pack_pair: copy rows x cols row-major FP16/BF16 operands with arbitrary
//    (element) alignment into 16-byte aligned rows x ld buffers, zero-filling the
//    padding columns -- A and B in one launch.  Used when an operand cannot be
//    described by a TMA tensor map (base not 16-byte aligned, or a row pitch that
//    is not a multiple of 16 bytes).
//  * tf32_prepare: both TF32 operands in one launch -- the rounded A copy and
//    the rounded, transposed B -- so the GEMM that follows (launched as its
//    programmatic dependent) overlaps its start-up with this pass.
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

// One launch for both TF32 operands.  Blocks [0, a_blocks) write the rounded A
// (m x k, row-major) into a_dst (m x lda, zero in columns k..lda-1); the other
// blocks write the rounded transpose of B (k x n, row-major) into b_dst (n x ldb,
// K-major, zero in columns k..ldb-1), in 64 x 64 tiles through shared memory
// with 16-byte global loads and stores on both sides.  lda and ldb are multiples
// of 4 and the destinations 16-byte aligned.  B goes K-major because the tensor
// core reads MN-major TF32 operands only in a 32-byte-atom swizzle; rounding and
// transposing in the same pass costs no extra traffic.
struct Tf32Prep {
    const float *a;
    float *a_dst;
    const float *b;
    float *b_dst;
    int64_t m, k, n, lda, ldb;
    int a_vec;     // A rows are 16-byte aligned and lda == k: one flat float4 stream
    int b_vec;     // B rows are 16-byte aligned (n % 4 == 0, aligned base)
    int a_blocks;  // blocks that work on A (may be 0 when A needs no copy)
};

constexpr int TP_TILE = 64;

__global__ void __launch_bounds__(256) tf32_prepare_kernel(const Tf32Prep p)
{
    __shared__ float tile[TP_TILE][TP_TILE + 1];
    wait_for_prior_grid();
    allow_next_grid();
    const int tid = threadIdx.x;
    if (static_cast<int>(blockIdx.x) < p.a_blocks) {
        const int64_t stride = static_cast<int64_t>(p.a_blocks) * 256;
        if (p.a_vec) {
            // Four independent 16-byte loads in flight per thread per iteration.
            const float4 *src = reinterpret_cast<const float4 *>(p.a);
            float4 *dst = reinterpret_cast<float4 *>(p.a_dst);
            const int64_t count4 = p.m * p.k / 4;
            for (int64_t base = static_cast<int64_t>(blockIdx.x) * 256 + tid; base < count4; base += 4 * stride) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (base + u * stride < count4)
                        v[u] = src[base + u * stride];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (base + u * stride < count4) {
                        v[u].x = round_tf32_rne(v[u].x);
                        v[u].y = round_tf32_rne(v[u].y);
                        v[u].z = round_tf32_rne(v[u].z);
                        v[u].w = round_tf32_rne(v[u].w);
                        dst[base + u * stride] = v[u];
                    }
                }
            }
        } else {
            const int64_t total = p.m * p.lda;
            for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + tid; i < total; i += stride) {
                const int64_t r = i / p.lda, col = i % p.lda;
                p.a_dst[i] = col < p.k ? round_tf32_rne(p.a[r * p.k + col]) : 0.0f;
            }
        }
        return;
    }
    const int64_t n_tiles = (p.n + TP_TILE - 1) / TP_TILE;
    const int64_t k_tiles = (p.ldb + TP_TILE - 1) / TP_TILE;
    const int64_t b_blocks = static_cast<int64_t>(gridDim.x) - p.a_blocks;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) - p.a_blocks; t < n_tiles * k_tiles; t += b_blocks) {
        const int64_t k0 = (t / n_tiles) * TP_TILE, n0 = (t % n_tiles) * TP_TILE;
        // Load: thread -> rows k0 + tid/16 + 16i, columns n0 + 4 (tid % 16) .. +3.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int kk = tid / 16 + 16 * i, c = (tid % 16) * 4;
            const int64_t gk = k0 + kk, gn = n0 + c;
            float v[4];
            if (p.b_vec && gk < p.k && gn + 3 < p.n) {
                const float4 x = *reinterpret_cast<const float4 *>(p.b + gk * p.n + gn);
                v[0] = x.x;
                v[1] = x.y;
                v[2] = x.z;
                v[3] = x.w;
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    v[q] = (gk < p.k && gn + q < p.n) ? p.b[gk * p.n + gn + q] : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
                tile[kk][c + q] = round_tf32_rne(v[q]);
        }
        __syncthreads();
        // Store: thread -> output row n0 + tid/16 + 16i, columns k0 + 4 (tid % 16) .. +3.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int nn = tid / 16 + 16 * i, kc = (tid % 16) * 4;
            const int64_t gn = n0 + nn, gk = k0 + kc;
            if (gn < p.n && gk < p.ldb)
                *reinterpret_cast<float4 *>(p.b_dst + gn * p.ldb + gk) =
                    make_float4(tile[kc][nn], tile[kc + 1][nn], tile[kc + 2][nn], tile[kc + 3][nn]);
        }
        __syncthreads();
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
