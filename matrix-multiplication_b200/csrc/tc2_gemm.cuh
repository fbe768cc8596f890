// CTA-pair (cta_group::2) variant of the tcgen05 GEMM: one 2-CTA cluster computes
// a 256 x 256 output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256).
//
// Split of the tile across the pair (rank r = %cluster_ctarank, 0 = leader):
//   * A: CTA r stages rows [m0 + 128 r, m0 + 128 r + 128) of the K slice;
//   * B: CTA r stages columns [n0 + 128 r, n0 + 128 r + 128);
//   * D: CTA r's TMEM holds output rows m0 + 128 r .. +127, all 256 columns.
// Both CTAs keep their operands at the same shared-memory offsets; the leader's
// descriptors name its own copy and the tensor cores of the pair read both.
// Each SM therefore stages and reads 32 KB per 256 x 256 x 64 step instead of
// 48 KB per 128 x 256 x 64 in the single-CTA kernel, which is what lets the
// pair run closer to the tensor-core rate.
//
// Synchronisation (all waits bounded, see ptx.cuh):
//   full[s]   leader only; the leader's producer arms it with both CTAs' bytes,
//             both CTAs' TMA loads complete on it (cta_group::2 loads).
//   empty[s]  in both CTAs; one multicast tcgen05.commit from the leader's MMA
//             thread arrives on both (two separate commits per stage cost ~10 %
//             of tensor-pipe time in the issue loop).
//   accf[i]   in both CTAs; committed the same way when accumulator i is done.
//   acce[i]   leader only; one arrive per epilogue warp of both CTAs (8).
// Warp roles and the epilogue are those of the single-CTA kernel (tc_gemm.cuh).
// No load uses cluster multicast: every CTA fetches its own tiles.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace b200 {

constexpr int TC2_BM = 256;                 // rows per pair tile
constexpr int TC2_BN = 256;                 // columns per pair tile
constexpr int TC2_HALF = 128;               // rows (A) / columns (B) staged per CTA
constexpr int TC2_STAGES = 6;
constexpr int TC2_A_STAGE = TC2_HALF * TC_ROW_BYTES;   // 16 KB
constexpr int TC2_B_STAGE = TC2_HALF * TC_ROW_BYTES;   // 16 KB
constexpr int TC2_SMEM_BYTES =
    1024 + TC2_STAGES * (TC2_A_STAGE + TC2_B_STAGE) + TC_EPI_BYTES + TC_BAR_BYTES;

template <int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
tc2_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, const TcParams p)
{
    constexpr bool kTF32 = FMT == kFmtTF32;
    constexpr int kElem = kTF32 ? 4 : 2;
    constexpr int kBK = TC_ROW_BYTES / kElem;          // K elements per stage (64 or 32)
    constexpr int kMmaK = 32 / kElem;                  // K per instruction (16 or 8)
    constexpr int kMmasPerStage = kBK / kMmaK;         // 4
    constexpr int kNB = TC_ROW_BYTES / kElem;          // MN-major B box width (64)
    constexpr int kBBoxes = TC2_HALF / kNB;            // 2 boxes per CTA half (MN-major B)
    constexpr uint32_t kBBoxBytes = kBK * TC_ROW_BYTES;
    constexpr bool kBKMajor = kTF32;
    constexpr uint32_t kIdesc = tc_instr_desc(FMT, kBKMajor, TC2_BM, TC2_BN);
    constexpr uint32_t kStageTx = 2u * (TC2_A_STAGE + TC2_B_STAGE);   // both CTAs

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t s_a = base;
    const uint32_t s_b = s_a + TC2_STAGES * TC2_A_STAGE;
    const uint32_t s_epi = s_b + TC2_STAGES * TC2_B_STAGE;
    const uint32_t s_bar = s_epi + TC_EPI_BYTES;
    auto full_bar = [&](int s) { return s_bar + 8u * s; };
    auto empty_bar = [&](int s) { return s_bar + 8u * (TC2_STAGES + s); };
    auto accf_bar = [&](int i) { return s_bar + 8u * (2 * TC2_STAGES + i); };
    auto acce_bar = [&](int i) { return s_bar + 8u * (2 * TC2_STAGES + 2 + i); };
    const uint32_t drain_bar = s_bar + 8u * (2 * TC2_STAGES + 4);
    const uint32_t tmem_slot = s_bar + 8u * (2 * TC2_STAGES + 5);
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_cta_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC2_STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(accf_bar(i), 1);
            mbar_init(acce_bar(i), 8);
        }
        mbar_init(drain_bar, 1);
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&map_a);
        tma_prefetch_map(&map_b);
        if (!p.c_direct)
            tma_prefetch_map(&map_c);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TC_TMEM_COLUMNS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    // Both CTAs' barriers are initialised before either CTA signals the other.
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot_ptr);
    wait_for_prior_grid();
    allow_next_grid();

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t filled = 0, fill_parity = 0;
            bool ok = true;
            const uint32_t leader_full0 = map_to_cta(full_bar(0), 0);
            for (int tile = pair; ok && tile < p.num_tiles; tile += pairs) {
                int mb, nb;
                tc_tile_coords(tile, p, mb, nb);
                const int a_row = mb * TC2_BM + static_cast<int>(rank) * TC2_HALF;
                const int b_col = nb * TC2_BN + static_cast<int>(rank) * TC2_HALF;
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
                        report_status(kStatusLoadTimeout);
                        ok = false;
                        break;
                    }
                    const uint32_t fb = leader_full0 + 8u * stage;
                    if (leader)
                        mbar_arrive_expect_tx(full_bar(stage), kStageTx);
                    tma_load_2d_pair(s_a + stage * TC2_A_STAGE, &map_a, fb, kb * kBK, a_row);
                    if constexpr (kBKMajor) {
                        tma_load_2d_pair(s_b + stage * TC2_B_STAGE, &map_b, fb, kb * kBK, b_col);
                    } else {
#pragma unroll
                        for (int j = 0; j < kBBoxes; ++j)
                            tma_load_2d_pair(s_b + stage * TC2_B_STAGE + j * kBBoxBytes, &map_b, fb, b_col + j * kNB,
                                             kb * kBK);
                    }
                    filled |= 1u << stage;
                    fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == TC2_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (leader) {
                for (int s = 0; s < TC2_STAGES; ++s)
                    if ((filled >> s) & 1u)
                        if (!mbar_wait(full_bar(s), (fill_parity >> s) & 1u))
                            report_status(kStatusDrainTimeout);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            // Loop-invariant descriptor halves: only the start-address field (bits 0-13,
            // address >> 4) moves between stages and K slices, so the issue loop adds.
            const uint64_t a_desc0 = smem_desc_sw128(s_a, 16, 1024);
            const uint64_t b_desc0 = kBKMajor ? smem_desc_sw128(s_b, 16, 1024) : smem_desc_sw128(s_b, kBBoxBytes, 1024);
            constexpr uint64_t kADescStage = TC2_A_STAGE >> 4;
            constexpr uint64_t kBDescStage = TC2_B_STAGE >> 4;
            constexpr uint64_t kADescK = 32 >> 4;
            constexpr uint64_t kBDescK = kBKMajor ? (32 >> 4) : ((kMmaK * TC_ROW_BYTES) >> 4);
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < p.num_tiles; tile += pairs) {
                if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u)) {
                    report_status(kStatusMmaTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TC2_BN);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase)) {
                        report_status(kStatusMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage) * kADescStage;
                    const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage) * kBDescStage;
#pragma unroll
                    for (int kk = 0; kk < kMmasPerStage; ++kk)
                        tc_mma_pair<kTF32>(d_tmem, a_desc + kk * kADescK, b_desc + kk * kBDescK, kIdesc,
                                      (kb | kk) != 0 ? 1u : 0u);
                    // Free this stage in both CTAs (one multicast commit).
                    tc_commit_pair_both(empty_bar(stage), 3);
                    if (++stage == TC2_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                tc_commit_pair_both(accf_bar(acc), 3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            tc_commit_pair(drain_bar);
            if (!mbar_wait(drain_bar, 0))
                report_status(kStatusDrainTimeout);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t stores = 0;
        for (int tile = pair; tile < p.num_tiles; tile += pairs) {
            int mb, nb;
            tc_tile_coords(tile, p, mb, nb);
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(accf_bar(acc), acc_phase) ? 1 : 0;
            ok = epilogue_all(__shfl_sync(0xffffffffu, ok, 0));
            if (!ok) {
                if (lane == 0)
                    report_status(kStatusEpilogueTimeout);
                break;
            }
            tc_fence_after();
            const int tile_row0 = mb * TC2_BM + static_cast<int>(rank) * TC2_HALF;   // first row of this CTA's part of the tile
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * TC2_BN);
#pragma unroll 1
            for (int chunk = 0; chunk < TC2_BN / 32; ++chunk) {
                uint32_t v[32];
                tmem_load_32cols(t_row + chunk * 32, v);
                if (chunk == TC2_BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(acce_bar(acc), 0));
                }
                const int col0 = nb * TC2_BN + chunk * 32;
                if (col0 >= p.n || tile_row0 >= p.m)      // the same for all four warps
                    continue;
                if (!p.c_direct) {
                    // One 128-row x 32-column box per chunk, filled by all four warps and
                    // stored by one thread: a quarter of the TMA operations of per-warp boxes.
                    const uint32_t box = s_epi + (stores & 1u) * (4 * TC_EPI_BOX);
                    const bool issuer = warp == 2 && lane == 0;
                    if (issuer)
                        bulk_wait_group_read<1>();        // the store that last read this buffer
                    epilogue_sync();
                    const int r = quarter * 32 + lane;
                    const uint32_t row_addr = box + r * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_shared_v4(row_addr + ((j ^ (r & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                     v[4 * j + 3]);
                    fence_proxy_async_shared();
                    epilogue_sync();
                    if (issuer) {
                        tma_store_2d(&map_c, box, col0, tile_row0);
                        bulk_commit_group();
                    }
                    ++stores;
                } else {
                    // C is not TMA-compatible: the same shared-memory box, written out one
                    // row per warp instruction (lane = column) with bounds-checked stores.
                    const uint32_t box = s_epi + (stores & 1u) * (4 * TC_EPI_BOX);
                    epilogue_sync();
                    const int r = quarter * 32 + lane;
                    const uint32_t row_addr = box + r * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_shared_v4(row_addr + ((j ^ (r & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                     v[4 * j + 3]);
                    epilogue_sync();
                    const float *box_f = reinterpret_cast<const float *>(smem_raw + (box - raw));
                    const int gcol = col0 + lane;
                    for (int rr = quarter; rr < TC_BM; rr += 4) {
                        const int grow = tile_row0 + rr;
                        if (grow < p.m && gcol < p.n)
                            p.c[static_cast<size_t>(grow) * p.n + gcol] =
                                box_f[rr * 32 + (((lane >> 2) ^ (rr & 7)) << 2) + (lane & 3)];
                    }
                    ++stores;
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (warp == 2 && lane == 0)
            bulk_wait_group_read<0>();     // shared memory free; the writes complete with the grid
        __syncwarp();
    }

    // Neither CTA releases TMEM before the pair's last MMA and both epilogues are done.
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TC_TMEM_COLUMNS);
    }
}

} // namespace b200
