// CTA-pair (cta_group::2) variant of the tcgen05 GEMM: one 2-CTA cluster computes
// a 256 x BN output tile (BN = 256 or 512) with tcgen05.mma.cta_group::2
// instructions of M = 256, N = 256 (BN / 256 of them per K step).
//
// Split of the tile across the pair (rank r = %cluster_ctarank, 0 = leader):
//   * A: CTA r stages rows [m0 + 128 r, m0 + 128 r + 128) of the K slice;
//   * B: for each 256-column half h of the tile, CTA r stages columns
//     [n0 + 256 h + 128 r, +128);
//   * D: CTA r's TMEM holds output rows m0 + 128 r .. +127, all BN columns
//     (TMEM column c = output column n0 + c).
// Both CTAs keep their operands at the same shared-memory offsets; the leader's
// descriptors name its own copy and the tensor cores of the pair read both.
//
// Operand bytes an SM stages per K block against its MMA cycles decide the rate:
// BN = 256 stages 32 KB per 512 cycles (64 B/cycle, more than the ~55 B/cycle an
// SM takes in from L2, so the tensor pipe idles ~10 %), BN = 512 stages 48 KB per
// 1024 cycles (48 B/cycle).  BN = 256 double-buffers its accumulator in TMEM (2 x
// 256 columns); BN = 512 fills all 512 columns with one accumulator, so the
// accumulator is handed over in two column halves.  In the last kDefer K blocks
// of a tile the MMA thread issues the column 0-255 MMAs first and commits that
// half, so the epilogue reads it while the column 256-511 MMAs of those blocks
// run; the next tile starts on columns 0-255 and holds back its column 256-511
// MMAs of the first kDefer K blocks (their stages stay resident) until the
// epilogue has read those columns too.  The K order of every sum is unchanged,
// so both widths give the same bits (1-3 deferred blocks measured alike).
//
// Synchronisation (all waits bounded, see ptx.cuh; the producers' waits for a
// freed stage keep the fixed limit, so that when the MMA thread gives up both
// CTAs of the pair stop issuing at the same stage and the leader's drain of its
// full barriers covers every copy either CTA issued):
//   full[s]   leader only; the leader's producer arms it with both CTAs' bytes,
//             both CTAs' TMA loads complete on it (cta_group::2 loads).
//   empty[s]  in both CTAs; one multicast tcgen05.commit from the leader's MMA
//             thread arrives on both (two separate commits per stage cost ~10 %
//             of tensor-pipe time in the issue loop).
//   accf[i]   in both CTAs; committed the same way when accumulator i is done
//             (BN = 512: accf[0] only).
//   acce[i]   leader only; one arrive per epilogue warp of both CTAs (8) when
//             accumulator i (BN = 512: column half i) has been read.
// Warp roles and the epilogue are those of the single-CTA kernel (tc_gemm.cuh).
// No load uses cluster multicast: every CTA fetches its own tiles.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace b200 {

constexpr int TC2_BM = 256;                 // rows per pair tile
constexpr int TC2_BN = 256;                 // columns per pair tile (narrow kernel)
constexpr int TC2W_BN = 512;                // columns per pair tile (wide kernel)
constexpr int TC2_HALF = 128;               // rows (A) / columns of a B half staged per CTA
constexpr int TC2_A_STAGE = TC2_HALF * TC_ROW_BYTES;   // 16 KB

template <int BN>
struct Tc2Tile {
    static_assert(BN == 256 || BN == 512, "pair tile width");
    static constexpr int kHalves = BN / 256;                        // N = 256 MMAs per K step
    static constexpr int kBStage = kHalves * TC2_HALF * TC_ROW_BYTES;   // 16 or 32 KB
    static constexpr int kStages = BN == 256 ? 6 : 4;
    static constexpr int kAccs = BN == 256 ? 2 : 1;                 // TMEM accumulators of BN columns
    static constexpr int kSmem = 1024 + kStages * (TC2_A_STAGE + kBStage) + TC_EPI_BYTES + TC_BAR_BYTES;
};
constexpr int TC2_STAGES = Tc2Tile<TC2_BN>::kStages;
constexpr int TC2_SMEM_BYTES = Tc2Tile<TC2_BN>::kSmem;
static_assert(Tc2Tile<TC2W_BN>::kSmem <= 227 * 1024, "wide pair tile exceeds shared memory");

template <int FMT, int BN = TC2_BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
tc2_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, const TcParams p)
{
    using Tile = Tc2Tile<BN>;
    constexpr int kStages = Tile::kStages;
    constexpr int kHalves = Tile::kHalves;
    constexpr int kBStage = Tile::kBStage;
    constexpr int kAccs = Tile::kAccs;
    constexpr int kDefer = 2;     // BN = 512: K blocks at each end of a tile run on one column half first
    static_assert(kDefer >= 1 && kDefer < kStages, "deferred K blocks must leave the producer a stage");
    constexpr bool kTF32 = FMT == kFmtTF32;
    constexpr int kElem = kTF32 ? 4 : 2;
    constexpr int kBK = TC_ROW_BYTES / kElem;          // K elements per stage (64 or 32)
    constexpr int kMmaK = 32 / kElem;                  // K per instruction (16 or 8)
    constexpr int kMmasPerStage = kBK / kMmaK;         // 4
    constexpr int kNB = TC_ROW_BYTES / kElem;          // MN-major B box width (64)
    constexpr int kBBoxes = TC2_HALF / kNB;            // 2 boxes per CTA half (MN-major B)
    constexpr uint32_t kBBoxBytes = kBK * TC_ROW_BYTES;
    constexpr uint32_t kIdesc = tc_instr_desc(FMT, false, TC2_BM, 256);   // B MN-major in every format
    constexpr uint32_t kBHalfBytes = TC2_HALF * TC_ROW_BYTES;         // one 128-column B half of a CTA
    constexpr uint32_t kStageTx = 2u * (TC2_A_STAGE + kBStage);       // both CTAs

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t s_a = base;
    const uint32_t s_b = s_a + kStages * TC2_A_STAGE;
    const uint32_t s_epi = s_b + kStages * kBStage;
    const uint32_t s_bar = s_epi + TC_EPI_BYTES;
    auto full_bar = [&](int s) { return s_bar + 8u * s; };
    auto empty_bar = [&](int s) { return s_bar + 8u * (kStages + s); };
    auto accf_bar = [&](int i) { return s_bar + 8u * (2 * kStages + i); };
    auto acce_bar = [&](int i) { return s_bar + 8u * (2 * kStages + 2 + i); };
    const uint32_t drain_bar = s_bar + 8u * (2 * kStages + 4);
    const uint32_t tmem_slot = s_bar + 8u * (2 * kStages + 5);
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_cta_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
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
                const int b_col = nb * BN + static_cast<int>(rank) * TC2_HALF;
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
#pragma unroll
                    for (int h = 0; h < kHalves; ++h) {
                        const uint32_t s_bh = s_b + stage * kBStage + h * kBHalfBytes;
#pragma unroll
                        for (int j = 0; j < kBBoxes; ++j)
                            tma_load_2d_pair(s_bh + j * kBBoxBytes, &map_b, fb, b_col + h * 256 + j * kNB, kb * kBK);
                    }
                    filled |= 1u << stage;
                    fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (leader) {
                for (int s = 0; s < kStages; ++s)
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
            const uint64_t b_desc0 = smem_desc_mn<kTF32>(s_b, kBBoxBytes);
            constexpr uint64_t kADescStage = TC2_A_STAGE >> 4;
            constexpr uint64_t kBDescStage = kBStage >> 4;
            constexpr uint64_t kBDescHalf = kBHalfBytes >> 4;
            constexpr uint64_t kADescK = 32 >> 4;
            constexpr uint64_t kBDescK = (kMmaK * TC_ROW_BYTES) >> 4;
            // The MMAs of one K block for one 256-column half of the accumulator.
            auto issue_half = [&](uint32_t d_tmem, int s, int h, int kb) {
                const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(s) * kADescStage;
                const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(s) * kBDescStage + h * kBDescHalf;
#pragma unroll
                for (int kk = 0; kk < kMmasPerStage; ++kk)
                    tc_mma_pair<kTF32>(d_tmem + static_cast<uint32_t>(h * 256), a_desc + kk * kADescK,
                                       b_desc + kk * kBDescK, kIdesc, (kb | kk) != 0 ? 1u : 0u);
            };
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < p.num_tiles; tile += pairs) {
                if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, p.wait_limit_ns)) {
                    report_status(kStatusMmaTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                const int nkb = p.num_k_blocks;
                bool upper_live = false;              // BN = 512: the epilogue has read columns 256-511
                int pending = 0, pending_stage = 0;   // BN = 512: K blocks whose column 256-511 MMAs wait
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.wait_limit_ns)) {
                        report_status(kStatusMmaTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_half(d_tmem, stage, 0, kb);
                    if constexpr (kHalves == 1) {
                        // Free this stage in both CTAs (one multicast commit).
                        tc_commit_pair_both(empty_bar(stage), 3);
                    } else {
                        if (kb == nkb - 1)
                            tc_commit_pair_both(accf_bar(0), 3);    // columns 0-255 complete
                        if (upper_live && kb < nkb - kDefer) {
                            issue_half(d_tmem, stage, 1, kb);
                            tc_commit_pair_both(empty_bar(stage), 3);
                        } else {
                            // The first kDefer K blocks (columns 256-511 still being read)
                            // and the last kDefer (columns 0-255 finish first, so their
                            // epilogue overlaps these MMAs) wait; then catch up, oldest
                            // first, and free their stages.
                            if (pending++ == 0)
                                pending_stage = stage;
                            if (kb == nkb - 1 || (!upper_live && kb == kDefer - 1)) {
                                if (!upper_live) {
                                    if (!mbar_wait(acce_bar(1), acc_phase ^ 1u, p.wait_limit_ns)) {
                                        report_status(kStatusMmaTimeout);
                                        ok = false;
                                        break;
                                    }
                                    tc_fence_after();
                                    upper_live = true;
                                }
                                int s = pending_stage;
                                for (int j = kb - pending + 1; j <= kb; ++j) {
                                    issue_half(d_tmem, s, 1, j);
                                    tc_commit_pair_both(empty_bar(s), 3);
                                    if (++s == kStages)
                                        s = 0;
                                }
                                pending = 0;
                            }
                        }
                    }
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                tc_commit_pair_both(accf_bar(kHalves == 1 ? acc : 1), 3);
                if (++acc == kAccs) {
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
        // All four epilogue warps wait for accumulator (half) i to be complete.
        auto wait_accf = [&](int i) {
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(accf_bar(i), acc_phase, p.wait_limit_ns) ? 1 : 0;
            ok = epilogue_all(__shfl_sync(0xffffffffu, ok, 0));
            if (!ok && lane == 0)
                report_status(kStatusEpilogueTimeout);
            tc_fence_after();
            return ok != 0;
        };
        bool ok = true;
        int failed_tile = -1;     // the first tile not finished (the same in all four warps)
        for (int tile = pair; ok && tile < p.num_tiles; tile += pairs) {
            int mb, nb;
            tc_tile_coords(tile, p, mb, nb);
            if (!wait_accf(kAccs == 2 ? acc : 0)) {
                failed_tile = tile;
                break;
            }
            const int tile_row0 = mb * TC2_BM + static_cast<int>(rank) * TC2_HALF;   // first row of this CTA's part of the tile
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int chunk = 0; chunk < BN / 32; ++chunk) {
                if (kAccs == 1 && chunk == 8 && !(ok = wait_accf(1))) {   // BN = 512: columns 256-511
                    failed_tile = tile;
                    break;
                }
                uint32_t v[32];
                tmem_load_32cols(t_row + chunk * 32, v);
                if (chunk % 8 == 7) {
                    // Accumulator `acc` (BN = 256) or column half chunk / 8 (BN = 512) read.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(acce_bar(kAccs == 2 ? acc : chunk / 8), 0));
                }
                const int col0 = nb * BN + chunk * 32;
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
            if (++acc == kAccs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (warp == 2 && lane == 0) {
            if (failed_tile >= 0)
                bulk_wait_group<0>();      // the stored boxes are in C before the NaN below
            else
                bulk_wait_group_read<0>(); // shared memory free; the writes complete with the grid
        }
        __syncwarp();
        if (failed_tile >= 0) {
            // This CTA's rows of every tile from the first unfinished one on.
            epilogue_sync();
            for (int tile = failed_tile; tile < p.num_tiles; tile += pairs) {
                int mb, nb;
                tc_tile_coords(tile, p, mb, nb);
                fill_nan(p.c, p.m, p.n, mb * TC2_BM + static_cast<int>(rank) * TC2_HALF, TC2_HALF, nb * BN, BN,
                         quarter, 4, lane);
            }
        }
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
