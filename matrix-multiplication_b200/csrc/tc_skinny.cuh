// Skinny GEMM (m <= 64): C = A * B computed as C^T = B^T * A^T on the tensor cores.
//
// With only a handful of rows the GEMM is HBM-bound on B (16 x 8192 x 8192 BF16
// reads 134 MB of B for 2.1 GFLOP).  Putting N on the MMA's 128-row side keeps
// the tensor core busy on useful work and lets each CTA stream a 128-column slab
// of B in 256-byte row segments:
//   * MMA "A" operand = B^T (128 columns n x one K block per stage), read straight
//     from row-major B as the MN-major operand: two 64-column TMA boxes for
//     FP16/BF16 (128-byte swizzle), four 32-column boxes for TF32 (32-byte-atom
//     swizzle, rounded to TF32 by the TFLOAT32 loads).
//   * MMA "B" operand = A^T (NP rows m x 64 k, K-major): NP = m rounded up to 16,
//     32 or 64.
//   * TMEM: 128 lanes (n) x NP columns (m), two accumulators.
//   * Epilogue: each warp loads 16 columns (m) of its 32 lanes (n) and writes, per
//     m, 32 consecutive floats of C's row m (one 128-byte store per warp per row).
//   * Split K when there are too few 128-column slabs to occupy the GPU: a
//     launch with gridDim.z = S > 1 forms clusters of (1, 1, S), one slab per
//     cluster; CTA z streams K blocks [z*ceil(nk/S), (z+1)*ceil(nk/S)), writes its
//     128 x NP FP32 partial into its idle ring, bulk-copies the rows (columns n)
//     [j*128/S, (j+1)*128/S) to CTA j, and sums the S partials of its own rows in
//     the fixed order 0..S-1 (deterministic, no zeroing of C, no atomics).
// Warp roles and bounded waits as in tc_gemm.cuh.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace b200 {

constexpr int SK_BM = 128;           // columns of C per tile (MMA M)
constexpr int SK_B_ROWS = 32;        // k-rows per TMA box of B^T

template <int NP>
struct SkTile {
    static_assert(NP == 16 || NP == 32 || NP == 64, "padded row count");
    static constexpr int kAStage = SK_BM * TC_ROW_BYTES;   // B^T slab: 16 KB
    static constexpr int kBStage = NP * TC_ROW_BYTES;      // A^T rows: 2, 4 or 8 KB
    static constexpr int kStages = NP == 64 ? 9 : 10;      // 144-160 KB of B in flight
    static constexpr int kSmem = 1024 + kStages * (kAStage + kBStage) + TC_BAR_BYTES;
    static constexpr uint32_t kTmemColumns = 2 * NP < 32 ? 32 : 2 * NP;
};

struct SkParams {
    int m, n, k;
    int num_n_tiles;          // 128-column slabs of C
    int num_k_blocks;         // K blocks per split (all of them when gridDim.z == 1)
    int total_k_blocks;
    float *c;
    unsigned long long wait_limit_ns;   // limit of the progress waits (ptx.cuh)
};

template <int FMT, int NP>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_skinny_kernel(const __grid_constant__ CUtensorMap map_bt, const __grid_constant__ CUtensorMap map_at,
                 const SkParams p)
{
    using Tile = SkTile<NP>;
    constexpr bool kTF32 = FMT == kFmtTF32;
    constexpr int kElem = kTF32 ? 4 : 2;
    constexpr int kBK = TC_ROW_BYTES / kElem;
    constexpr int kMmaK = 32 / kElem;
    constexpr int kMmasPerStage = kBK / kMmaK;
    // B^T (the MMA's A side) is read MN-major from B's rows in every format.
    constexpr int kNB = TC_ROW_BYTES / kElem;              // columns per MN-major box (64)
    constexpr uint32_t kBoxBytes = kBK * TC_ROW_BYTES;     // 8 KB per MN-major box
    constexpr int kStages = Tile::kStages;
    constexpr int kAStage = Tile::kAStage;
    constexpr int kBStage = Tile::kBStage;
    constexpr uint32_t kTmemColumns = Tile::kTmemColumns;
    // Operand "A" = B^T: MN-major (FP16/BF16) or K-major (TF32); operand "B" = A^T: K-major.
    constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(FMT) << 7) | (static_cast<uint32_t>(FMT) << 10) |
                                (1u << 15) | (0u << 16) |
                                (static_cast<uint32_t>(NP >> 3) << 17) | (static_cast<uint32_t>(SK_BM >> 4) << 24);

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t s_a = base;                              // B^T slabs
    const uint32_t s_b = s_a + kStages * kAStage;          // A^T rows
    const uint32_t s_bar = s_b + kStages * kBStage;
    auto full_bar = [&](int s) { return s_bar + 8u * s; };
    auto empty_bar = [&](int s) { return s_bar + 8u * (kStages + s); };
    auto accf_bar = [&](int i) { return s_bar + 8u * (2 * kStages + i); };
    auto acce_bar = [&](int i) { return s_bar + 8u * (2 * kStages + 2 + i); };
    const uint32_t drain_bar = s_bar + 8u * (2 * kStages + 4);
    const uint32_t tmem_slot = s_bar + 8u * (2 * kStages + 5);
    const uint32_t recv_bar = s_bar + 8u * (2 * kStages + 6);   // split K: partial rows received
    const uint32_t fail_flag = s_bar + 8u * (2 * kStages + 7);  // 1 once a progress wait of this CTA ran out
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));
    volatile uint32_t *fail_flag_ptr = reinterpret_cast<volatile uint32_t *>(smem_raw + (fail_flag - raw));
    // Split K: 128 x NP FP32 partial rows (n) padded to NP + 4 floats, then the
    // S-1 received slices, in the idle operand ring.
    constexpr uint32_t kPartialPitch = (NP + 4) * 4;
    constexpr uint32_t kPartialBytes = SK_BM * kPartialPitch;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int splits = static_cast<int>(gridDim.z);
    const int split = static_cast<int>(blockIdx.z);
    const int kb0 = split * p.num_k_blocks;
    const int kb1 = min(kb0 + p.num_k_blocks, p.total_k_blocks);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(accf_bar(i), 1);
            mbar_init(acce_bar(i), 128);
        }
        mbar_init(drain_bar, 1);
        mbar_init(recv_bar, 1);
        *fail_flag_ptr = 0u;
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&map_bt);
        tma_prefetch_map(&map_at);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemColumns);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot_ptr);
    wait_for_prior_grid();
    allow_next_grid();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t filled = 0, fill_parity = 0;
            bool ok = true;
            for (int nt = blockIdx.x; ok && nt < p.num_n_tiles; nt += gridDim.x) {
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.wait_limit_ns)) {
                        report_status(kStatusLoadTimeout);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), kAStage + kBStage);
                    // Boxes of 32 k-rows, the column boxes of each 32 rows issued together:
                    // the two 128-byte halves of a 256-byte row segment are requested close
                    // together (FP16/BF16: 3-4 % faster than whole-stage boxes, measured;
                    // 8- and 16-row boxes were slower).
#pragma unroll
                    for (int r = 0; r < kBK; r += SK_B_ROWS)
#pragma unroll
                        for (int j = 0; j < SK_BM / kNB; ++j)
                            tma_load_2d(s_a + stage * kAStage + j * kBoxBytes + r * TC_ROW_BYTES, &map_bt,
                                        full_bar(stage), nt * SK_BM + j * kNB, kb * kBK + r);
                    tma_load_2d(s_b + stage * kBStage, &map_at, full_bar(stage), kb * kBK, 0);
                    filled |= 1u << stage;
                    fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int s = 0; s < kStages; ++s)
                if ((filled >> s) & 1u)
                    if (!mbar_wait(full_bar(s), (fill_parity >> s) & 1u))
                        report_status(kStatusDrainTimeout);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            const uint64_t a_desc0 = smem_desc_mn<kTF32>(s_a, kBoxBytes);
            const uint64_t b_desc0 = smem_desc_sw128(s_b, 16, 1024);
            constexpr uint64_t kADescStage = kAStage >> 4;
            constexpr uint64_t kBDescStage = kBStage >> 4;
            constexpr uint64_t kADescK = (kMmaK * TC_ROW_BYTES) >> 4;
            constexpr uint64_t kBDescK = 32 >> 4;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int nt = blockIdx.x; ok && nt < p.num_n_tiles; nt += gridDim.x) {
                if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, p.wait_limit_ns)) {
                    report_status(kStatusMmaTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * NP);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.wait_limit_ns)) {
                        report_status(kStatusMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage) * kADescStage;
                    const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage) * kBDescStage;
#pragma unroll
                    for (int kk = 0; kk < kMmasPerStage; ++kk)
                        tc_mma<kTF32>(d_tmem, a_desc + kk * kADescK, b_desc + kk * kBDescK, kIdesc,
                                      (kb > kb0 || kk > 0) ? 1u : 0u);
                    tc_commit(empty_bar(stage));
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                if (kb0 < kb1)
                    tc_commit(accf_bar(acc));
                else
                    mbar_arrive(accf_bar(acc));     // an empty split: its partial is zero
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            tc_commit(drain_bar);
            if (!mbar_wait(drain_bar, 0))
                report_status(kStatusDrainTimeout);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;                 // TMEM lanes = columns n of C
        int acc = 0;
        uint32_t acc_phase = 0;
        int failed_tile = -1;     // this warp's first slab whose accumulator never arrived
        for (int nt = blockIdx.x; nt < p.num_n_tiles; nt += gridDim.x) {
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(accf_bar(acc), acc_phase, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) {
                    report_status(kStatusEpilogueTimeout);
                    *fail_flag_ptr = 1u;
                }
                failed_tile = nt;
                break;
            }
            tc_fence_after();
            if (splits > 1)
                break;     // one slab; its partial is exchanged below
            const int col = nt * SK_BM + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * NP);
#pragma unroll 1
            for (int chunk = 0; chunk < NP / 16; ++chunk) {
                uint32_t v[16];
                tmem_load_16cols(t_row + chunk * 16, v);
                if (chunk == NP / 16 - 1) {
                    tc_fence_before();
                    mbar_arrive(acce_bar(acc));
                }
                if (col < p.n) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int row = chunk * 16 + j;
                        if (row < p.m)
                            p.c[static_cast<size_t>(row) * p.n + col] = __uint_as_float(v[j]);
                    }
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        __syncwarp();
        if (failed_tile >= 0 && splits == 1) {
            // This warp's 32 columns of C (all m rows) in every slab from the failed one on.
            for (int nt = failed_tile; nt < p.num_n_tiles; nt += gridDim.x)
                fill_nan(p.c, p.m, p.n, 0, p.m, nt * SK_BM + quarter * 32, 32, 0, 1, lane);
        }
    }

    if (splits > 1 && kPartialBytes + static_cast<uint32_t>(splits - 1) * (kPartialBytes / splits) >
                          static_cast<uint32_t>(kStages * (kAStage + kBStage))) {
        if (threadIdx.x == 0)
            report_status(kStatusEpilogueTimeout);     // a launch the host never makes
    } else if (splits > 1) {
        const int rows = SK_BM / splits;                 // columns n of the slab summed by each CTA
        const uint32_t slice_bytes = static_cast<uint32_t>(rows) * kPartialPitch;
        const int nt = static_cast<int>(blockIdx.x);
        if (threadIdx.x == 0)
            mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(splits - 1) * slice_bytes);
        cluster_sync_all();     // every CTA of the cluster is past its main loop: rings idle
        // A CTA whose progress wait ran out has no valid partial: the columns of
        // every CTA of the cluster become NaN.
        const bool any_failed = cluster_any_failed(fail_flag, splits);
        if (warp >= 2) {
            const int quarter = warp & 3;
            const uint32_t row_addr = s_a + static_cast<uint32_t>(quarter * 32 + lane) * kPartialPitch;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
            for (int chunk = 0; chunk < NP / 16; ++chunk) {
                uint32_t v[16];
                if (kb0 < kb1) {
                    tmem_load_16cols(t_row + chunk * 16, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        v[j] = 0u;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    st_shared_v4(row_addr + (chunk * 16 + 4 * j) * 4, v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                 v[4 * j + 3]);
            }
            fence_proxy_async_shared();     // the bulk copies below read these stores
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int j = 0; j < splits; ++j) {
                if (j == split)
                    continue;
                const uint32_t slot = static_cast<uint32_t>(split < j ? split : split - 1);
                bulk_copy_to_cluster(map_to_cta(s_a + kPartialBytes + slot * slice_bytes, static_cast<uint32_t>(j)),
                                     s_a + static_cast<uint32_t>(j) * slice_bytes, slice_bytes,
                                     map_to_cta(recv_bar, static_cast<uint32_t>(j)));
            }
        }
        int received = 1;
        if (lane == 0)
            received = mbar_wait(recv_bar, 0) ? 1 : 0;
        received = __shfl_sync(0xffffffffu, received, 0);
        if (!received && lane == 0)
            report_status(kStatusDrainTimeout);
        if (any_failed || !received)
            fill_nan(p.c, p.m, p.n, 0, p.m, nt * SK_BM + split * rows, rows, warp, TC_THREADS / 32, lane);
        const uint8_t *ring = smem_raw + (s_a - raw);
        for (int idx = threadIdx.x; received && !any_failed && idx < p.m * rows; idx += TC_THREADS) {
            const int row = idx / rows, rl = idx % rows;    // C row (m), column offset within the slice
            const uint32_t offset = static_cast<uint32_t>(rl) * kPartialPitch + static_cast<uint32_t>(row) * 4;
            float sum = 0.0f;
#pragma unroll
            for (int src = 0; src < 8; ++src) {
                if (src < splits) {
                    const uint32_t base_off =
                        src == split ? static_cast<uint32_t>(split) * slice_bytes
                                     : kPartialBytes + static_cast<uint32_t>(src < split ? src : src - 1) * slice_bytes;
                    const float v = *reinterpret_cast<const float *>(ring + base_off + offset);
                    sum = src == 0 ? v : sum + v;
                }
            }
            const int col = nt * SK_BM + split * rows + rl;
            if (col < p.n)
                p.c[static_cast<size_t>(row) * p.n + col] = sum;
        }
        // No CTA leaves while a copy into it (or out of it) may be in flight.
        cluster_sync_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemColumns);
    }
}

} // namespace b200
