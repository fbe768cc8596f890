// Pedantic FP32 GEMM on the FFMA pipe: C = A * B with FP32 multiply-add only
// (no TF32 anywhere), row-major, any m, k, n >= 1 and any 4-byte alignment.
//
// Replaces the reference's FP32 kernels (matmul_tiled_fp32 / matmul_register_fp32
// in src/matmul.cu:73-195 and matmul_warp_fp32 in src/matmul_custom.cuh:85-156)
// with one register-blocked kernel:
//   * 128 x 128 output tile per 256-thread block, K step 16, two blocks per SM;
//   * each thread owns an 8 x 8 micro-tile split into 2 x 2 groups of 4 x 4 that
//     are 64 rows / columns apart, so every shared-memory operand read is a
//     conflict-free float4 and each warp's B reads are two 128-byte rows;
//   * A is stored transposed (k-major) in shared memory, B as is;
//   * the next K tile is fetched from global memory into registers while the
//     current one is multiplied out of a double-buffered shared tile (one
//     barrier per K step);
//   * float4 global loads/stores when rows are 16-byte aligned, guarded scalar
//     accesses otherwise (offset base pointers, odd k or n, partial tiles).
#pragma once

#include <cstdint>

namespace b200 {

constexpr int FF_BM = 128;
constexpr int FF_BN = 128;
constexpr int FF_BK = 16;
constexpr int FF_THREADS = 256;

template <bool VEC_A, bool VEC_B, bool VEC_C>
__global__ void __launch_bounds__(FF_THREADS, 2)
ffma_gemm_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c, int m,
                 int n, int k)
{
    __shared__ __align__(16) float as[2][FF_BK][FF_BM];
    __shared__ __align__(16) float bs[2][FF_BK][FF_BN];

    const int tid = threadIdx.x;
    const int tx = tid & 15;                 // column group
    const int ty = tid >> 4;                 // row group
    // Global -> shared mapping.  A: each thread loads 8 consecutive k of one row
    // (a warp covers 32 rows with the same k offset: conflict-free transposed stores).
    const int a_row = tid & 127;
    const int a_k = (tid >> 7) * 8;
    // B: each thread loads float4 at columns 4*(tid%16) and 64 + 4*(tid%16) of row tid/16.
    const int b_k = tid >> 4;
    const int b_col = (tid & 15) * 4;
    const int num_kt = (k + FF_BK - 1) / FF_BK;

    for (int block_m = blockIdx.y; block_m * FF_BM < m; block_m += gridDim.y) {
        for (int block_n = blockIdx.x; block_n * FF_BN < n; block_n += gridDim.x) {
            const int m0 = block_m * FF_BM;
            const int n0 = block_n * FF_BN;
            const int grow = m0 + a_row;
            const bool a_row_ok = grow < m;
            const float *a_ptr = a + static_cast<size_t>(a_row_ok ? grow : 0) * k;

            float ra[8];
            float rb[8];
            auto fetch = [&](int kt) {
                const int kbase = kt * FF_BK;
                // A: 8 values a[grow][kbase + a_k + 0..7]
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int kk = kbase + a_k + 4 * h;
                    if (VEC_A && a_row_ok && kk + 3 < k) {
                        const float4 v = *reinterpret_cast<const float4 *>(a_ptr + kk);
                        ra[4 * h] = v.x;
                        ra[4 * h + 1] = v.y;
                        ra[4 * h + 2] = v.z;
                        ra[4 * h + 3] = v.w;
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            ra[4 * h + q] = (a_row_ok && kk + q < k) ? a_ptr[kk + q] : 0.0f;
                    }
                }
                // B: row kbase + b_k, columns n0 + b_col + {0..3} and n0 + 64 + b_col + {0..3}
                const int krow = kbase + b_k;
                const bool k_ok = krow < k;
                const float *b_ptr = b + static_cast<size_t>(k_ok ? krow : 0) * n;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = n0 + b_col + 64 * h;
                    if (VEC_B && k_ok && col + 3 < n) {
                        const float4 v = *reinterpret_cast<const float4 *>(b_ptr + col);
                        rb[4 * h] = v.x;
                        rb[4 * h + 1] = v.y;
                        rb[4 * h + 2] = v.z;
                        rb[4 * h + 3] = v.w;
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            rb[4 * h + q] = (k_ok && col + q < n) ? b_ptr[col + q] : 0.0f;
                    }
                }
            };
            auto stash = [&](int buf) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    as[buf][a_k + q][a_row] = ra[q];
                *reinterpret_cast<float4 *>(&bs[buf][b_k][b_col]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
                *reinterpret_cast<float4 *>(&bs[buf][b_k][64 + b_col]) =
                    make_float4(rb[4], rb[5], rb[6], rb[7]);
            };

            float acc[8][8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    acc[i][j] = 0.0f;

            fetch(0);
            stash(0);
            __syncthreads();
            int buf = 0;
            for (int kt = 0; kt < num_kt; ++kt) {
                if (kt + 1 < num_kt)
                    fetch(kt + 1);
#pragma unroll
                for (int kk = 0; kk < FF_BK; ++kk) {
                    const float4 a0 = *reinterpret_cast<const float4 *>(&as[buf][kk][ty * 4]);
                    const float4 a1 = *reinterpret_cast<const float4 *>(&as[buf][kk][64 + ty * 4]);
                    const float4 b0 = *reinterpret_cast<const float4 *>(&bs[buf][kk][tx * 4]);
                    const float4 b1 = *reinterpret_cast<const float4 *>(&bs[buf][kk][64 + tx * 4]);
                    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                }
                if (kt + 1 < num_kt)
                    stash(buf ^ 1);
                __syncthreads();
                buf ^= 1;
            }

#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
                if (row >= m)
                    continue;
                float *c_row = c + static_cast<size_t>(row) * n;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = n0 + tx * 4 + 64 * h;
                    if (VEC_C && col + 3 < n) {
                        *reinterpret_cast<float4 *>(c_row + col) =
                            make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (col + q < n)
                                c_row[col + q] = acc[i][4 * h + q];
                    }
                }
            }
        }
    }
}

} // namespace b200
