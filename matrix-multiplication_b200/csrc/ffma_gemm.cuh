// Pedantic FP32 GEMM on the FFMA pipe: C = A * B with FP32 multiply-add only
// (no TF32 anywhere), row-major, any m, k, n >= 1 and any 4-byte alignment.
//
// Replaces the reference's FP32 kernels (matmul_tiled_fp32 / matmul_register_fp32
// in src/matmul.cu:73-195 and matmul_warp_fp32 in src/matmul_custom.cuh:85-156)
// with one register-blocked kernel:
//   * a 3- or 4-stage cp.async pipeline feeds shared memory straight from global
//     memory (no register staging, one barrier per 16- or 32-deep K tile): 16-byte
//     copies when A and B rows are 16-byte aligned (k % 4 == 0, n % 4 == 0,
//     aligned bases), 4-byte copies otherwise (offset bases, odd k or n); partial
//     tiles are zero-filled by cp.async's source-size operand;
//   * A stays row-major in shared memory (rows padded by 4 floats) and is read as
//     float4 along k, so one A fragment load serves four k-slices; B is read as
//     float4 along n;
//   * the multiply-adds are packed FP32x2 FMAs (__ffma2_rn: two IEEE
//     round-to-nearest FMAs per issued instruction), so instruction issue does
//     not cap the FMA pipe;
//   * float4 stores of C when its rows are 16-byte aligned, guarded scalar
//     stores otherwise.
#pragma once

#include <cstdint>

#include "pack.cuh"
#include "ptx.cuh"

namespace b200 {

constexpr int FF_BM = 128;
constexpr int FF_BN = 128;
constexpr int FF_THREADS = 256;

// Split K: a launch with gridDim.z = S > 1 must form clusters of (1, 1, S).  The
// S CTAs of a cluster compute the same output tile over S consecutive slices of
// the K tiles, stage their FP32 partial tiles in their own shared memory, and
// after a cluster barrier CTA r sums rows [r*BM/S, (r+1)*BM/S) of all S partials
// through distributed shared memory in the fixed order 0, 1, ..., S-1 and stores
// them: more CTAs for outputs too small to fill the GPU, no workspace in global
// memory, and a result that does not depend on timing.
//
// The output tile is BM x BN, each thread owning an RM x RN micro-tile, so the
// block has (BM/RM) x (BN/RN) threads: 128 x 128 with 8 x 8 per thread (256
// threads) for large problems and 32 x 32 with 4 x 4 (64 threads) so that
// smaller outputs still spread over every SM.  A thread's rows are ty, ty + TY,
// ... (TY = BM/RM): the threads of a warp then read A rows BK + 4 floats apart,
// which fall in distinct banks.  Its columns come in groups of four, 4*TX apart (TX = BN/RN), so a warp's
// B reads are contiguous 16-byte vectors.
constexpr int FA_MODEL_BK = 16;                          // K granularity of the launch-plan model

template <int BM, int BN, int RM, int RN>
struct FaTile {
    static constexpr int kTX = BN / RN;                  // threads along a row of the tile
    static constexpr int kTY = BM / RM;
    static constexpr int kThreads = kTX * kTY;
    static constexpr int kVecN = RN >= 4 ? 4 : 2;        // floats per B fragment read / C store
    static_assert(BM % RM == 0 && BN % RN == 0 && RN % kVecN == 0 && RN >= 2, "micro-tile");
    static_assert(kThreads % 32 == 0 && kThreads <= 256, "thread count");
    // K depth and ring length per tile: the 128 x 128 tile takes 32-deep stages
    // (half the barriers per FMA; two blocks still fit an SM), smaller tiles
    // 16-deep ones (four stages from 64 x 64 up, three below).
    static constexpr int kBK = BM * BN >= 128 * 128 ? 32 : 16;
    static constexpr int kStages = BM * BN >= 128 * 128 ? 3 : BM * BN >= 64 * 64 ? 4 : 3;
    static constexpr int kALd = kBK + 4;                 // padded row of the A tile (floats)
    static constexpr int kAStage = BM * kALd;            // floats
    static constexpr int kBStage = kBK * BN;             // floats
    static constexpr int kPipeBytes = kStages * (kAStage + kBStage) * 4;
    static constexpr int kPartialBytes = BM * BN * 4;    // split-K partial tile
    static constexpr int kSmemBytes = kPipeBytes > kPartialBytes ? kPipeBytes : kPartialBytes;
    static constexpr int kAChunks = BM * kBK / 4;        // 16-byte copies per stage
    static constexpr int kBChunks = kBK * BN / 4;
    // Blocks per SM the register budget is sized for: 128 registers for an
    // 8 x 8 micro-tile, fewer for the small ones.
    static constexpr int kRegs = RM * RN >= 64 ? 128 : RM * RN >= 16 ? 80 : 40;
    static constexpr int kMinBlocks = 65536 / (kThreads * kRegs) > 8 ? 8 : 65536 / (kThreads * kRegs);

    __device__ static __forceinline__ int row(int ty, int i) { return ty + kTY * i; }
    __device__ static __forceinline__ int col(int tx, int j)   // j: first of a vector group
    {
        return (j / kVecN) * (kVecN * kTX) + tx * kVecN + (j % kVecN);
    }
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

// 4-byte copy with zero fill when !valid (unaligned operands).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, bool valid)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Store V consecutive outputs of one row starting at column `col` (bounds-checked
// against n; one vector store when VEC and the whole vector is inside).
template <int V, bool VEC>
__device__ __forceinline__ void store_row_vec(float *c_row, int col, int n, const float *v)
{
    if (VEC && col + V - 1 < n) {
        if constexpr (V == 4)
            *reinterpret_cast<float4 *>(c_row + col) = make_float4(v[0], v[1], v[2], v[3]);
        else
            *reinterpret_cast<float2 *>(c_row + col) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int q = 0; q < V; ++q)
            if (col + q < n)
                c_row[col + q] = v[q];
    }
}

// TF32_ROUND: each K tile is rounded to TF32 (nearest even) in shared memory once
// it has landed -- the TF32 GEMM of small problems on the FFMA pipe: a product of
// two TF32 values is exact in FP32, so the result has the same products as the
// tensor-core path, accumulated in FP32.
template <int BM, int BN, int RM, int RN, bool VEC_AB, bool VEC_C, bool TF32_ROUND = false>
__global__ void __launch_bounds__(FaTile<BM, BN, RM, RN>::kThreads, FaTile<BM, BN, RM, RN>::kMinBlocks)
ffma_gemm_async_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c, int m,
                       int n, int k)
{
    using T = FaTile<BM, BN, RM, RN>;
    constexpr int BK = T::kBK, STAGES = T::kStages, A_LD = T::kALd;
    constexpr int kVecN = T::kVecN;
    constexpr int kThreads = T::kThreads;
    extern __shared__ __align__(16) float fa_smem[];
    float *as = fa_smem;                                    // [stage][BM][A_LD]
    float *bs = fa_smem + STAGES * T::kAStage;           // [stage][BK][BN]
    const uint32_t as_addr = static_cast<uint32_t>(__cvta_generic_to_shared(as));
    const uint32_t bs_addr = static_cast<uint32_t>(__cvta_generic_to_shared(bs));

    wait_for_prior_grid();
    allow_next_grid();
    const int tid = threadIdx.x;
    const int tx = tid % T::kTX;
    const int ty = tid / T::kTX;
    // K tiles [kt_begin, kt_begin + num_kt) of this CTA's split (possibly none).
    const int splits = static_cast<int>(gridDim.z);
    const int split = static_cast<int>(blockIdx.z);
    const int total_kt = (k + BK - 1) / BK;
    const int kt_per_split = (total_kt + splits - 1) / splits;
    const int kt_begin = split * kt_per_split;
    const int num_kt = max(0, min(total_kt, kt_begin + kt_per_split) - kt_begin);

    for (int block_m = blockIdx.y; block_m * BM < m; block_m += gridDim.y) {
        for (int block_n = blockIdx.x; block_n * BN < n; block_n += gridDim.x) {
            const int m0 = block_m * BM;
            const int n0 = block_n * BN;

            // Tile kt (of this split) -> stage s: A is BM rows x BK/4 chunks, B is BK rows x BN/4 chunks.
            auto issue = [&](int kt, int s) {
#pragma unroll
                for (int h = 0; h < (T::kAChunks + kThreads - 1) / kThreads; ++h) {
                    const int chunk = tid + kThreads * h;
                    if (T::kAChunks % kThreads == 0 || chunk < T::kAChunks) {
                        const int row = chunk / (BK / 4), kq = chunk % (BK / 4);
                        const int grow = m0 + row, gk = (kt_begin + kt) * BK + kq * 4;
                        const uint32_t dst = as_addr + (s * T::kAStage + row * A_LD + kq * 4) * 4;
                        if constexpr (VEC_AB) {
                            const bool ok = grow < m && gk < k;
                            cp_async16(dst, ok ? a + static_cast<size_t>(grow) * k + gk : a, ok);
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const bool ok = grow < m && gk + e < k;
                                cp_async4(dst + 4 * e, ok ? a + static_cast<size_t>(grow) * k + gk + e : a, ok);
                            }
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < (T::kBChunks + kThreads - 1) / kThreads; ++h) {
                    const int chunk = tid + kThreads * h;
                    if (T::kBChunks % kThreads == 0 || chunk < T::kBChunks) {
                        const int row = chunk / (BN / 4), cq = chunk % (BN / 4);
                        const int gk = (kt_begin + kt) * BK + row, gcol = n0 + cq * 4;
                        const uint32_t dst = bs_addr + (s * T::kBStage + row * BN + cq * 4) * 4;
                        if constexpr (VEC_AB) {
                            const bool ok = gk < k && gcol < n;
                            cp_async16(dst, ok ? b + static_cast<size_t>(gk) * n + gcol : b, ok);
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const bool ok = gk < k && gcol + e < n;
                                cp_async4(dst + 4 * e, ok ? b + static_cast<size_t>(gk) * n + gcol + e : b, ok);
                            }
                        }
                    }
                }
            };

            // acc[i][p] holds outputs (row i, columns 2p and 2p + 1).
            float2 acc[RM][RN / 2];
#pragma unroll
            for (int i = 0; i < RM; ++i)
#pragma unroll
                for (int j = 0; j < RN / 2; ++j)
                    acc[i][j] = make_float2(0.0f, 0.0f);

#pragma unroll
            for (int s = 0; s < STAGES - 1; ++s) {
                if (s < num_kt)
                    issue(s, s);
                cp_async_commit();
            }
            for (int kt = 0; kt < num_kt; ++kt) {
                cp_async_wait<STAGES - 2>();
                __syncthreads();
                const int next = kt + STAGES - 1;
                if (next < num_kt)
                    issue(next, next % STAGES);
                cp_async_commit();
                const float *at = as + (kt % STAGES) * T::kAStage;
                const float *bt = bs + (kt % STAGES) * T::kBStage;
                if constexpr (TF32_ROUND) {
                    // Round this stage in place once (every value is read by several threads).
                    float4 *stage_a = reinterpret_cast<float4 *>(as + (kt % STAGES) * T::kAStage);
                    float4 *stage_b = reinterpret_cast<float4 *>(bs + (kt % STAGES) * T::kBStage);
                    for (int i = tid; i < T::kAStage / 4 + T::kBStage / 4; i += kThreads) {
                        float4 *q = i < T::kAStage / 4 ? stage_a + i : stage_b + (i - T::kAStage / 4);
                        float4 v = *q;
                        v.x = round_tf32_rne(v.x);
                        v.y = round_tf32_rne(v.y);
                        v.z = round_tf32_rne(v.z);
                        v.w = round_tf32_rne(v.w);
                        *q = v;
                    }
                    __syncthreads();
                }
#pragma unroll
                for (int k4 = 0; k4 < BK; k4 += 4) {
                    float4 ar[RM];
#pragma unroll
                    for (int i = 0; i < RM; ++i)
                        ar[i] = *reinterpret_cast<const float4 *>(at + T::row(ty, i) * A_LD + k4);

#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        float2 bp[RN / 2];
#pragma unroll
                        for (int j = 0; j < RN; j += kVecN) {
                            const float *src = bt + (k4 + kk) * BN + T::col(tx, j);
                            if constexpr (kVecN == 4) {
                                const float4 v = *reinterpret_cast<const float4 *>(src);
                                bp[j / 2] = make_float2(v.x, v.y);
                                bp[j / 2 + 1] = make_float2(v.z, v.w);
                            } else {
                                bp[j / 2] = *reinterpret_cast<const float2 *>(src);
                            }
                        }
#pragma unroll
                        for (int i = 0; i < RM; ++i) {
                            const float av = kk == 0 ? ar[i].x : kk == 1 ? ar[i].y : kk == 2 ? ar[i].z : ar[i].w;
                            const float2 ai = make_float2(av, av);
#pragma unroll
                            for (int j = 0; j < RN / 2; ++j)
                                acc[i][j] = __ffma2_rn(ai, bp[j], acc[i][j]);
                        }
                    }
                }
            }
            cp_async_wait<0>();
            __syncthreads();

            if (splits == 1) {
#pragma unroll
                for (int i = 0; i < RM; ++i) {
                    const int row = m0 + T::row(ty, i);
                    if (row >= m)
                        continue;
                    float *c_row = c + static_cast<size_t>(row) * n;
#pragma unroll
                    for (int j = 0; j < RN; j += kVecN) {
                        const int col = n0 + T::col(tx, j);
                        float v[kVecN];
#pragma unroll
                        for (int q = 0; q < kVecN; q += 2) {
                            v[q] = acc[i][(j + q) / 2].x;
                            v[q + 1] = acc[i][(j + q) / 2].y;
                        }
                        store_row_vec<kVecN, VEC_C>(c_row, col, n, v);
                    }
                }
                continue;
            }

            // Split K: partial tile (row-major, BM x BN) into this CTA's shared memory.
#pragma unroll
            for (int i = 0; i < RM; ++i) {
                float *p_row = fa_smem + T::row(ty, i) * BN;
#pragma unroll
                for (int j = 0; j < RN; j += kVecN) {
                    if constexpr (kVecN == 4)
                        *reinterpret_cast<float4 *>(p_row + T::col(tx, j)) =
                            make_float4(acc[i][j / 2].x, acc[i][j / 2].y, acc[i][j / 2 + 1].x, acc[i][j / 2 + 1].y);
                    else
                        *reinterpret_cast<float2 *>(p_row + T::col(tx, j)) = acc[i][j / 2];
                }
            }
            cluster_sync_all();
            {
                const uint32_t part_addr = static_cast<uint32_t>(__cvta_generic_to_shared(fa_smem));
                const int rows = BM / splits;                  // this CTA's slice of the tile
                const int row0 = split * rows;
                for (int idx = tid; idx < rows * (BN / 4); idx += kThreads) {
                    const int r = row0 + idx / (BN / 4), c4 = (idx % (BN / 4)) * 4;
                    const uint32_t offset = static_cast<uint32_t>((r * BN + c4) * 4);
                    float4 sum = ld_shared_cluster_f4(map_to_cta(part_addr + offset, 0));
                    for (int src = 1; src < splits; ++src) {
                        const float4 v = ld_shared_cluster_f4(map_to_cta(part_addr + offset, src));
                        sum.x += v.x;
                        sum.y += v.y;
                        sum.z += v.z;
                        sum.w += v.w;
                    }
                    if (m0 + r < m) {
                        const float v[4] = {sum.x, sum.y, sum.z, sum.w};
                        store_row_vec<4, VEC_C>(c + static_cast<size_t>(m0 + r) * n, n0 + c4, n, v);
                    }
                }
            }
            // No CTA reuses (or leaves) its shared memory while another still reads it.
            cluster_sync_all();
        }
    }
}

} // namespace b200
