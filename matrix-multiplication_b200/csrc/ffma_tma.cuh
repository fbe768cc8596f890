// Pedantic FP32 GEMM on the FFMA pipe with TMA-staged operands: C = A * B with
// FP32 multiply-add only (no TF32 anywhere), row-major, for operands whose base
// addresses and row pitches are 16-byte aligned (k % 4 == 0, n % 4 == 0).
//
// Same arithmetic as ffma_gemm_async_kernel's 128 x 128 tile (src/matmul_custom.cuh:
// 85-156 is the reference kernel it replaces): 256 threads, 8 x 8 outputs per thread,
// packed FP32x2 FMAs, each output's sum over k in increasing k order.  What differs is
// the staging: one thread issues one TMA box of A (128 rows x 32 k) and four of B
// (32 k x 32 columns each) per 32-deep K tile into a 3-stage ring (two CTAs per
// SM), completion counted on an mbarrier per stage, instead of every thread
// issuing eight cp.async copies with their own address arithmetic per stage.
// The FMA loop, not the staging, bounds this kernel: the TMA form runs about 1 %
// faster than the cp.async one.
//
// Shared-memory layout (128-byte swizzle, 1024-byte aligned boxes): row r of an
// A box holds k = 0..31 of output row r as eight 16-byte chunks, chunk q stored at
// position q ^ (r & 7); row kk of a B box holds 32 columns the same way, chunk q at
// q ^ (kk & 7).  A thread's A rows are ty + 16 i, all with the same r & 7, so its
// float4 reads along k stay conflict-free; a warp's B reads cover whole 128-byte
// rows.  Out-of-range rows and columns of a box arrive as zeros, so partial tiles
// need no special case in the loop.
//
// Split K and waits: as ffma_gemm_async_kernel (clusters of (1, 1, S), fixed-order
// sum through distributed shared memory).  A wait for a stage is bounded by the
// launch's limit; when it runs out, every thread of the CTA stops together
// (__syncthreads_and), thread 0 waits (2 s at most) for the copies it issued, the
// status word is set and the CTA's unfinished outputs are written as NaN.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace b200 {

constexpr int FT_BM = 128, FT_BN = 128, FT_BK = 32;
constexpr int FT_THREADS = 256, FT_TX = 16, FT_TY = 16, FT_RM = 8, FT_RN = 8;
constexpr int FT_STAGES = 3;
constexpr int FT_A_BYTES = FT_BM * FT_BK * 4;        // 16 KB: 128 rows x 128 bytes
constexpr int FT_B_BOX = FT_BK * 32 * 4;             // 4 KB: 32 k-rows x 32 columns
constexpr int FT_STAGE_BYTES = FT_A_BYTES + 4 * FT_B_BOX;
constexpr int FT_BAR_BYTES = 64;
constexpr int FT_SMEM = 1024 + FT_STAGES * FT_STAGE_BYTES + FT_BAR_BYTES;
static_assert(FT_STAGES * FT_STAGE_BYTES >= FT_BM * FT_BN * 4, "split-K partial tile fits the ring");
static_assert(2 * FT_SMEM <= 228 * 1024, "two CTAs per SM");

struct FtParams {
    int m, n, k;
    float *c;
    unsigned long long wait_limit_ns;
};

template <bool VEC_C>
__global__ void __launch_bounds__(FT_THREADS, 2)
ffma_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const FtParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t s_bar = base + FT_STAGES * FT_STAGE_BYTES;
    auto full_bar = [&](int s) { return s_bar + 8u * static_cast<uint32_t>(s); };
    const uint32_t fail_flag = s_bar + 8u * FT_STAGES;
    volatile uint32_t *fail_flag_ptr = reinterpret_cast<volatile uint32_t *>(smem_raw + (fail_flag - raw));
    const float *ring = reinterpret_cast<const float *>(smem_raw + (base - raw));

    const int tid = threadIdx.x;
    const int tx = tid % FT_TX, ty = tid / FT_TX;
    const int splits = static_cast<int>(gridDim.z);
    const int split = static_cast<int>(blockIdx.z);
    const int total_kt = (p.k + FT_BK - 1) / FT_BK;
    const int kt_per_split = (total_kt + splits - 1) / splits;
    const int kt_begin = split * kt_per_split;
    const int num_kt = max(0, min(total_kt, kt_begin + kt_per_split) - kt_begin);

    if (tid == 0) {
        for (int s = 0; s < FT_STAGES; ++s)
            mbar_init(full_bar(s), 1);
        *fail_flag_ptr = 0u;
        fence_mbarrier_init();
        tma_prefetch_map(&map_a);
        tma_prefetch_map(&map_b);
    }
    __syncthreads();
    wait_for_prior_grid();
    allow_next_grid();

    // K tiles are numbered across this CTA's output tiles: tile `it` uses stage
    // it % FT_STAGES in phase (it / FT_STAGES) & 1.
    int issued = 0, consumed = 0;
    bool failed = false;
    for (int block_m = blockIdx.y; block_m * FT_BM < p.m; block_m += gridDim.y) {
        for (int block_n = blockIdx.x; block_n * FT_BN < p.n; block_n += gridDim.x) {
            const int m0 = block_m * FT_BM, n0 = block_n * FT_BN;
            if (failed) {
                // A wait of this CTA ran out: the rest of its tiles are NaN.
                fill_nan(p.c, p.m, p.n, m0, FT_BM, n0, FT_BN, tid / 32, FT_THREADS / 32, tid % 32);
                continue;
            }
            auto issue = [&](int kt) {     // thread 0: K tile kt of this split into the next stage
                const int s = issued % FT_STAGES;
                const uint32_t sa = base + static_cast<uint32_t>(s) * FT_STAGE_BYTES;
                const int kg = (kt_begin + kt) * FT_BK;
                mbar_arrive_expect_tx(full_bar(s), FT_STAGE_BYTES);
                tma_load_2d(sa, &map_a, full_bar(s), kg, m0);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    tma_load_2d(sa + FT_A_BYTES + j * FT_B_BOX, &map_b, full_bar(s), n0 + 32 * j, kg);
                ++issued;
            };
            if (tid == 0)
                for (int kt = 0; kt < FT_STAGES - 1 && kt < num_kt; ++kt)
                    issue(kt);

            float2 acc[FT_RM][FT_RN / 2];
#pragma unroll
            for (int i = 0; i < FT_RM; ++i)
#pragma unroll
                for (int j = 0; j < FT_RN / 2; ++j)
                    acc[i][j] = make_float2(0.0f, 0.0f);

            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = consumed % FT_STAGES;
                const int ok = mbar_wait(full_bar(s), static_cast<uint32_t>(consumed / FT_STAGES) & 1u,
                                         p.wait_limit_ns) ? 1 : 0;
                // Also: every thread is done with the stage the next copy overwrites.
                if (!__syncthreads_and(ok)) {
                    failed = true;
                    break;
                }
                if (tid == 0 && kt + FT_STAGES - 1 < num_kt)
                    issue(kt + FT_STAGES - 1);
                const float *as = ring + s * (FT_STAGE_BYTES / 4);
                const float *bs = as + FT_A_BYTES / 4;
                ++consumed;
                // A fragments four k deep (float4 along k): one shared-memory load serves
                // four k-slices.  Fully unrolled, this needs more than the 128 registers two
                // CTAs per SM allow and spills a little (88 bytes), yet it ran 1.1 % faster
                // than the cp.async kernel and 13 % faster than a rolled 2-deep loop that
                // spilled nothing (4096^3 and 8192^3, interleaved replays on one B200).
#pragma unroll
                for (int k4 = 0; k4 < FT_BK; k4 += 4) {
                    float4 ar[FT_RM];
#pragma unroll
                    for (int i = 0; i < FT_RM; ++i)
                        ar[i] = *reinterpret_cast<const float4 *>(as + (ty + FT_TY * i) * FT_BK +
                                                                  (((k4 >> 2) ^ (ty & 7)) << 2));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const int kr = k4 + kk;
                        float2 bp[FT_RN / 2];
#pragma unroll
                        for (int g = 0; g < 2; ++g) {      // columns g*64 + tx*4 .. +3
                            const int box = g * 2 + (tx >> 3);
                            const float4 v = *reinterpret_cast<const float4 *>(
                                bs + box * (FT_B_BOX / 4) + kr * 32 + (((tx & 7) ^ (kr & 7)) << 2));
                            bp[2 * g] = make_float2(v.x, v.y);
                            bp[2 * g + 1] = make_float2(v.z, v.w);
                        }
#pragma unroll
                        for (int i = 0; i < FT_RM; ++i) {
                            const float av = kk == 0 ? ar[i].x : kk == 1 ? ar[i].y : kk == 2 ? ar[i].z : ar[i].w;
                            const float2 ai = make_float2(av, av);
#pragma unroll
                            for (int j = 0; j < FT_RN / 2; ++j)
                                acc[i][j] = __ffma2_rn(ai, bp[j], acc[i][j]);
                        }
                    }
                }
            }
            if (failed) {
                if (tid == 0) {
                    // Copies already issued land before the CTA moves on or exits.
                    for (int it = consumed; it < issued; ++it)
                        if (!mbar_wait(full_bar(it % FT_STAGES), static_cast<uint32_t>(it / FT_STAGES) & 1u))
                            report_status(kStatusDrainTimeout);
                    report_status(kStatusLoadTimeout);
                    *fail_flag_ptr = 1u;
                }
                consumed = issued;
                __syncthreads();
                if (splits == 1)
                    fill_nan(p.c, p.m, p.n, m0, FT_BM, n0, FT_BN, tid / 32, FT_THREADS / 32, tid % 32);
            } else {
                __syncthreads();      // every thread is done reading the ring
            }

            if (splits == 1) {
                if (failed)
                    continue;
#pragma unroll
                for (int i = 0; i < FT_RM; ++i) {
                    const int row = m0 + ty + FT_TY * i;
                    if (row >= p.m)
                        continue;
                    float *c_row = p.c + static_cast<size_t>(row) * p.n;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        const int col = n0 + g * 64 + tx * 4;
                        const float v[4] = {acc[i][2 * g].x, acc[i][2 * g].y, acc[i][2 * g + 1].x,
                                            acc[i][2 * g + 1].y};
                        if (VEC_C && col + 3 < p.n) {
                            *reinterpret_cast<float4 *>(c_row + col) = make_float4(v[0], v[1], v[2], v[3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (col + q < p.n)
                                    c_row[col + q] = v[q];
                        }
                    }
                }
                continue;
            }

            // Split K: this CTA's partial tile (row-major 128 x 128) into its ring.
            float *partial = reinterpret_cast<float *>(smem_raw + (base - raw));
#pragma unroll
            for (int i = 0; i < FT_RM; ++i) {
                float *p_row = partial + (ty + FT_TY * i) * FT_BN;
#pragma unroll
                for (int g = 0; g < 2; ++g)
                    *reinterpret_cast<float4 *>(p_row + g * 64 + tx * 4) =
                        make_float4(acc[i][2 * g].x, acc[i][2 * g].y, acc[i][2 * g + 1].x, acc[i][2 * g + 1].y);
            }
            cluster_sync_all();
            {
                const bool any_failed = cluster_any_failed(fail_flag, splits);
                const uint32_t part_addr = base;
                const int rows = FT_BM / splits;           // this CTA's slice of the tile
                const int row0 = split * rows;
                if (any_failed) {
                    fill_nan(p.c, p.m, p.n, m0 + row0, rows, n0, FT_BN, tid / 32, FT_THREADS / 32, tid % 32);
                } else {
                    for (int idx = tid; idx < rows * (FT_BN / 4); idx += FT_THREADS) {
                        const int r = row0 + idx / (FT_BN / 4), c4 = (idx % (FT_BN / 4)) * 4;
                        const uint32_t offset = static_cast<uint32_t>((r * FT_BN + c4) * 4);
                        float4 sum = ld_shared_cluster_f4(map_to_cta(part_addr + offset, 0));
                        for (int src = 1; src < splits; ++src) {
                            const float4 v = ld_shared_cluster_f4(map_to_cta(part_addr + offset, src));
                            sum.x += v.x;
                            sum.y += v.y;
                            sum.z += v.z;
                            sum.w += v.w;
                        }
                        if (m0 + r < p.m) {
                            float *dst = p.c + static_cast<size_t>(m0 + r) * p.n + n0 + c4;
                            const float v[4] = {sum.x, sum.y, sum.z, sum.w};
                            if (VEC_C && n0 + c4 + 3 < p.n) {
                                *reinterpret_cast<float4 *>(dst) = sum;
                            } else {
                                for (int q = 0; q < 4 && n0 + c4 + q < p.n; ++q)
                                    dst[q] = v[q];
                            }
                        }
                    }
                }
            }
            // No CTA reuses (or leaves) its shared memory while another still reads it.
            cluster_sync_all();
            if (tid == 0)
                *fail_flag_ptr = 0u;      // the flag covers one tile of a split launch
            failed = false;
        }
    }
}

} // namespace b200
