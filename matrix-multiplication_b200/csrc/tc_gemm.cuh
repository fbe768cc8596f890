// Persistent warp-specialised tcgen05 GEMM: C (FP32, m x n) = A (m x k) * B (k x n),
// row-major, TF32 / FP16 / BF16 inputs, FP32 accumulation in tensor memory.
//
// Replaces the reference's matmul_wmma<T,BK> (src/matmul_custom.cuh:169-235),
// which staged scalars through shared memory into mma.sync fragments.  Here:
//
//   warp 0      TMA producer: one elected lane streams A (up to 128 x 128 B;
//               for m < 128 only the first m rows rounded up to 16, the MMA's
//               other rows hold stale data whose outputs are never stored) and
//               B (128 B-wide column blocks) boxes into a 4-stage ring with
//               128-byte swizzle, signalling a "full" mbarrier per stage.
//   warp 1      TMEM owner + MMA issuer: allocates 512 TMEM columns (two
//               128 x 256 FP32 accumulators) and one lane issues
//               tcgen05.mma (M=128, N=256, K=32 bytes) per K slice; a
//               tcgen05.commit frees each smem stage and publishes each
//               finished accumulator.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, stage them in a
//               swizzled 32 x 32 FP32 box per warp and TMA-store them (or, when C
//               is not TMA-compatible, store directly with bounds checks).
//               Runs one tile behind the MMA thanks to the two accumulators.
//
// A is K-major in shared memory.  B stays row-major (N contiguous), i.e. the
// MN-major operand form of the instruction descriptor, so neither operand is
// transposed in memory: FP16/BF16 boxes use the 128-byte swizzle, TF32 boxes
// the 128-byte swizzle with 32-byte atoms that an MN-major TF32 operand needs.
// TF32 operands are FP32 words in memory; the TMA loads of their TFLOAT32
// tensor maps round each to TF32 (nearest even) on the way in.  Tiles are
// visited persistently (tile += gridDim.x) in groups of `group_m` M-blocks so
// that concurrently running CTAs share A and B panels in L2.
//
// Split K (gridDim.z = S > 1, launched as clusters of (1, 1, S) with one tile per
// cluster, gridDim.x = num_tiles): CTA z of a cluster runs K blocks
// [z*ceil(nk/S), (z+1)*ceil(nk/S)) of the tile.  After a cluster barrier (every
// operand ring idle) it writes its accumulator into its ring, bulk-copies rows
// [j*128/S, (j+1)*128/S) into CTA j's shared memory (cp.async.bulk between the
// CTAs of the cluster), and sums the S partials of its own rows in the fixed
// order 0..S-1.  The partial and the S-1 received slices fit the ring plus the
// epilogue staging area: S <= 4 for 256-wide tiles, S <= 8 otherwise.  Few output tiles over a long K otherwise leave most SMs idle and
// the busy ones waiting on operand latency.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"

namespace b200 {

// Device status word: bit flags set by a kernel whose bounded wait gave up.
__device__ unsigned int g_device_status;

enum : unsigned int {
    kStatusLoadTimeout = 1u,
    kStatusMmaTimeout = 2u,
    kStatusEpilogueTimeout = 4u,
    kStatusDrainTimeout = 8u,
};

__device__ __forceinline__ void report_status(unsigned int flag)
{
    atomicOr(&g_device_status, flag);
}

// A kernel whose progress wait ran out writes NaN over every output element it
// did not finish, so that a later FP64 check of C fails loudly instead of
// passing over stale values: rows [row0, row0 + rows) x columns [col0, col0 +
// cols) of C, clipped to m x n, one warp per row (lanes along the columns).
__device__ __forceinline__ void fill_nan(float *c, int m, int n, int row0, int rows, int col0, int cols,
                                         int warp_index, int warps, int lane)
{
    const int row_end = min(m, row0 + rows), col_end = min(n, col0 + cols);
    const float nan = __int_as_float(0x7fc00000);
    for (int r = row0 + warp_index; r < row_end; r += warps)
        for (int col = col0 + lane; col < col_end; col += 32)
            c[static_cast<size_t>(r) * n + col] = nan;
}

// Whether any CTA of this cluster (ranks 0 .. ctas-1) set its failure flag (a
// 32-bit word at the same shared-memory offset in every CTA).  Only between two
// cluster barriers, while every CTA of the cluster is still running.
__device__ __forceinline__ bool cluster_any_failed(uint32_t flag, int ctas)
{
    uint32_t any = 0;
    for (int r = 0; r < ctas; ++r)
        any |= ld_shared_cluster_u32(map_to_cta(flag, static_cast<uint32_t>(r)));
    return any != 0;
}

enum TcFormat : int { kFmtF16 = 0, kFmtBF16 = 1, kFmtTF32 = 2 };

constexpr int TC_BM = 128;                  // rows per tile (TMEM lanes)
constexpr int TC_BN = 256;                  // columns per tile (TMEM columns per accumulator)
constexpr int TC_STAGES = 4;                // smem ring depth
constexpr int TC_THREADS = 192;             // 6 warps
constexpr int TC_ROW_BYTES = 128;           // one swizzle row = K-slice depth of a stage
constexpr int TC_A_STAGE = TC_BM * TC_ROW_BYTES;   // 16 KB
constexpr int TC_B_STAGE = TC_BN * TC_ROW_BYTES;   // 32 KB (BK rows x BN elements)
constexpr int TC_EPI_BOX = 32 * 32 * 4;            // 32 rows x 32 FP32 columns
constexpr int TC_EPI_BYTES = 4 * 2 * TC_EPI_BOX;   // 4 warps, double buffered
constexpr int TC_BAR_BYTES = 512;
constexpr int TC_SMEM_BYTES =
    1024 /* alignment slack */ + TC_STAGES * (TC_A_STAGE + TC_B_STAGE) + TC_EPI_BYTES + TC_BAR_BYTES;
constexpr uint32_t TC_TMEM_COLUMNS = 2 * TC_BN;

// Geometry of the single-CTA kernel for a tile width BN (256, 128 or 64) and an
// A stage of AROWS rows (128, or 32 for m <= 32): the narrower tiles give small
// and skinny problems more CTAs, and the smaller stages buy a deeper ring in the
// same ~225 KB of shared memory (16 stages, 128 KB of B in flight per SM, for
// the skinny, HBM-bound case).
template <int BN, int AROWS = 128>
struct TcTile {
    static_assert(BN == 256 || BN == 128 || BN == 64, "tile width");
    static_assert(AROWS == 128 || AROWS == 32, "A stage rows");
    static constexpr int kAStage = AROWS * TC_ROW_BYTES;
    static constexpr int kBStage = BN * TC_ROW_BYTES;
    static constexpr int kStages = AROWS == 32 ? 16 : BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static constexpr int kSmem = 1024 + kStages * (kAStage + kBStage) + TC_EPI_BYTES + TC_BAR_BYTES;
    static constexpr uint32_t kTmemColumns = 2 * BN;   // two accumulators
};

struct TcParams {
    int m, n, k;
    int num_m_blocks, num_n_blocks, num_k_blocks;
    int num_tiles;
    int group_m;     // M-blocks per raster group
    float *c;        // output (direct-store epilogue only)
    int c_direct;    // 1 when C cannot be written by TMA
    int a_box_rows;  // rows per A box (single-CTA kernel: m rounded up to 16 when m < 128)
    unsigned long long wait_limit_ns;   // limit of the progress waits (ptx.cuh)
};

// Instruction descriptor (kind::f16 / kind::tf32): FP32 accumulator (bits 4-5 = 1),
// A/B formats (bits 7-9, 10-12), A K-major (bit 15 = 0), B MN-major (bit 16 = 1)
// or K-major (0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t tc_instr_desc(int fmt, bool b_k_major, int mma_m = TC_BM, int mma_n = TC_BN)
{
    return (1u << 4) | (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |
           (0u << 15) | ((b_k_major ? 0u : 1u) << 16) | (static_cast<uint32_t>(mma_n >> 3) << 17) |
           (static_cast<uint32_t>(mma_m >> 4) << 24);
}

__device__ __forceinline__ void tc_tile_coords(int tile, const TcParams &p, int &mb, int &nb)
{
    const int per_group = p.group_m * p.num_n_blocks;
    const int group = tile / per_group;
    const int first_m = group * p.group_m;
    const int rows = min(p.num_m_blocks - first_m, p.group_m);
    const int local = tile - group * per_group;
    mb = first_m + local % rows;
    nb = local / rows;
}

template <int FMT, int BN, int AROWS = 128>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_c, const TcParams p)
{
    using Tile = TcTile<BN, AROWS>;
    constexpr int kStages = Tile::kStages;
    constexpr int kAStage = Tile::kAStage;
    constexpr int kBStage = Tile::kBStage;
    constexpr uint32_t kTmemColumns = Tile::kTmemColumns;
    constexpr bool kTF32 = FMT == kFmtTF32;
    constexpr int kElem = kTF32 ? 4 : 2;
    constexpr int kBK = TC_ROW_BYTES / kElem;          // K elements per stage (64 or 32)
    constexpr int kMmaK = 32 / kElem;                  // K per instruction (16 or 8)
    constexpr int kMmasPerStage = kBK / kMmaK;         // 4
    constexpr int kNB = TC_ROW_BYTES / kElem;          // B box width in elements (64 or 32)
    constexpr int kBBoxes = BN / kNB;                  // MN-major B boxes per stage
    constexpr uint32_t kBBoxBytes = kBK * TC_ROW_BYTES;  // bytes per B column block
    // B is read MN-major straight from its row-major rows (N contiguous) in every
    // format; TF32 in 32-byte-atom swizzled boxes (smem_desc_mn).
    constexpr uint32_t kIdesc = tc_instr_desc(FMT, false, TC_BM, BN);
    // Split K: this CTA's 128 x BN FP32 partial, then up to S-1 received row
    // slices, in the operand ring and the epilogue staging area behind it.
    constexpr uint32_t kPartialRowBytes = BN * 4;
    constexpr uint32_t kPartialBytes = TC_BM * kPartialRowBytes;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t s_a = base;
    const uint32_t s_b = s_a + kStages * kAStage;
    const uint32_t s_epi = s_b + kStages * kBStage;
    const uint32_t s_bar = s_epi + TC_EPI_BYTES;
    auto full_bar = [&](int s) { return s_bar + 8u * s; };
    auto empty_bar = [&](int s) { return s_bar + 8u * (kStages + s); };
    auto accf_bar = [&](int i) { return s_bar + 8u * (2 * kStages + i); };
    auto acce_bar = [&](int i) { return s_bar + 8u * (2 * kStages + 2 + i); };
    const uint32_t drain_bar = s_bar + 8u * (2 * kStages + 4);
    const uint32_t tmem_slot = s_bar + 8u * (2 * kStages + 5);
    const uint32_t recv_bar = s_bar + 8u * (2 * kStages + 6);   // split K: partial slices received
    const uint32_t fail_flag = s_bar + 8u * (2 * kStages + 7);  // 1 once a progress wait of this CTA ran out
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));
    volatile uint32_t *fail_flag_ptr = reinterpret_cast<volatile uint32_t *>(smem_raw + (fail_flag - raw));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // K blocks [kb_begin, kb_end) of this CTA's split (all of them when unsplit).
    const int splits = static_cast<int>(gridDim.z);
    const int kb_per_split = (p.num_k_blocks + splits - 1) / splits;
    const int kb_begin = static_cast<int>(blockIdx.z) * kb_per_split;
    const int kb_end = min(p.num_k_blocks, kb_begin + kb_per_split);
    const bool has_k = kb_begin < kb_end;

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
        tma_prefetch_map(&map_a);
        tma_prefetch_map(&map_b);
        if (!p.c_direct)
            tma_prefetch_map(&map_c);
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
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                int mb, nb;
                tc_tile_coords(tile, p, mb, nb);
                for (int kb = kb_begin; kb < kb_end; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.wait_limit_ns)) {
                        report_status(kStatusLoadTimeout);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), p.a_box_rows * TC_ROW_BYTES + kBStage);
                    tma_load_2d(s_a + stage * kAStage, &map_a, full_bar(stage), kb * kBK, mb * TC_BM);
#pragma unroll
                    for (int j = 0; j < kBBoxes; ++j)
                        tma_load_2d(s_b + stage * kBStage + j * kBBoxBytes, &map_b, full_bar(stage),
                                    nb * BN + j * kNB, kb * kBK);
                    filled |= 1u << stage;
                    fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Let every issued copy land before the CTA can exit.
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
            // Loop-invariant descriptor halves: only the start-address field (bits 0-13,
            // address >> 4) moves between stages and K slices, so the issue loop adds.
            const uint64_t a_desc0 = smem_desc_sw128(s_a, 16, 1024);
            const uint64_t b_desc0 = smem_desc_mn<kTF32>(s_b, kBBoxBytes);
            constexpr uint64_t kADescStage = kAStage >> 4;
            constexpr uint64_t kBDescStage = kBStage >> 4;
            constexpr uint64_t kADescK = 32 >> 4;
            constexpr uint64_t kBDescK = (kMmaK * TC_ROW_BYTES) >> 4;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, p.wait_limit_ns)) {
                    report_status(kStatusMmaTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = kb_begin; kb < kb_end; ++kb) {
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
                                      (kb != kb_begin || kk != 0) ? 1u : 0u);
                    tc_commit(empty_bar(stage));
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                if (has_k)
                    tc_commit(accf_bar(acc));
                else
                    mbar_arrive(accf_bar(acc));     // an empty split: its partial is zero
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // Every MMA issued above completes before TMEM is released.
            tc_commit(drain_bar);
            if (!mbar_wait(drain_bar, 0))
                report_status(kStatusDrainTimeout);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;               // TMEM lanes 32*quarter .. +31
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t stores = 0;
        int failed_tile = -1;     // the first tile whose accumulator never arrived (the same in all four warps)
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            int mb, nb;
            tc_tile_coords(tile, p, mb, nb);
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(accf_bar(acc), acc_phase, p.wait_limit_ns) ? 1 : 0;
            ok = epilogue_all(__shfl_sync(0xffffffffu, ok, 0));
            if (!ok) {
                if (lane == 0) {
                    report_status(kStatusEpilogueTimeout);
                    *fail_flag_ptr = 1u;
                }
                failed_tile = tile;
                break;
            }
            tc_fence_after();
            const int tile_row0 = mb * TC_BM;   // first row of this CTA's part of the tile
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
            if (splits > 1)
                break;     // one tile; its accumulator is pushed to the owning CTAs below
#pragma unroll 1
            for (int chunk = 0; chunk < BN / 32; ++chunk) {
                uint32_t v[32];
                tmem_load_32cols(t_row + chunk * 32, v);
                if (chunk == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(acce_bar(acc));
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
            if (++acc == 2) {
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
        if (failed_tile >= 0 && splits == 1) {
            epilogue_sync();
            for (int tile = failed_tile; tile < p.num_tiles; tile += gridDim.x) {
                int mb, nb;
                tc_tile_coords(tile, p, mb, nb);
                fill_nan(p.c, p.m, p.n, mb * TC_BM, TC_BM, nb * BN, BN, quarter, 4, lane);
            }
        }
    }

    if (splits > 1 && kPartialBytes + static_cast<uint32_t>(splits - 1) * (kPartialBytes / splits) >
                          static_cast<uint32_t>(kStages * (kAStage + kBStage) + TC_EPI_BYTES)) {
        if (threadIdx.x == 0)
            report_status(kStatusEpilogueTimeout);     // a launch the host never makes
    } else if (splits > 1) {
        // One tile per cluster.  Rows [j*rows, (j+1)*rows) of the tile are summed by
        // CTA j.  Every CTA writes its accumulator into its own ring as a row-major
        // partial (16-byte chunks XOR-swizzled by row), then the TMA engine copies
        // each row slice to the CTA that owns it, into slot [sender, skipping the
        // owner] behind the owner's partial; the owner adds the S slices in the
        // order 0..S-1.
        const int rows = TC_BM / splits;
        const uint32_t slice_bytes = static_cast<uint32_t>(rows) * kPartialRowBytes;
        const int z = static_cast<int>(blockIdx.z);
        if (threadIdx.x == 0)
            mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(splits - 1) * slice_bytes);
        cluster_sync_all();     // every CTA of the cluster is past its main loop: rings idle
        // A CTA whose progress wait ran out has no valid partial: the rows of
        // every CTA of the cluster become NaN.
        const bool any_failed = cluster_any_failed(fail_flag, splits);
        if (warp >= 2) {
            const int quarter = warp & 3;
            const int r = quarter * 32 + lane;
            const uint32_t row_addr = s_a + static_cast<uint32_t>(r) * kPartialRowBytes;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
            for (int chunk = 0; chunk < BN / 32; ++chunk) {
                uint32_t v[32];
                if (has_k) {
                    tmem_load_32cols(t_row + chunk * 32, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] = 0u;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    st_shared_v4(row_addr + (((chunk * 8 + j) ^ (r & 7)) << 4), v[4 * j], v[4 * j + 1],
                                 v[4 * j + 2], v[4 * j + 3]);
            }
            fence_proxy_async_shared();     // the bulk copies below read these stores
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int j = 0; j < splits; ++j) {
                if (j == z)
                    continue;
                const uint32_t slot = static_cast<uint32_t>(z < j ? z : z - 1);
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
        int mb, nb;
        tc_tile_coords(static_cast<int>(blockIdx.x), p, mb, nb);
        if (any_failed || !received)
            fill_nan(p.c, p.m, p.n, mb * TC_BM + z * rows, rows, nb * BN, BN, warp, TC_THREADS / 32, lane);
        const bool vec = !p.c_direct;
        const uint8_t *ring = smem_raw + (s_a - raw);
        for (int idx = threadIdx.x; received && !any_failed && idx < rows * (BN / 4); idx += TC_THREADS) {
            const int rl = idx / (BN / 4), q = idx % (BN / 4);
            const int r = z * rows + rl;                       // row within the tile
            const uint32_t offset = static_cast<uint32_t>(rl) * kPartialRowBytes +
                                    (static_cast<uint32_t>(q ^ (r & 7)) << 4);
            float4 part[8];
#pragma unroll
            for (int src = 0; src < 8; ++src) {
                if (src < splits) {
                    const uint32_t base_off = src == z ? static_cast<uint32_t>(z) * slice_bytes
                                                       : kPartialBytes + static_cast<uint32_t>(src < z ? src : src - 1) *
                                                                             slice_bytes;
                    part[src] = *reinterpret_cast<const float4 *>(ring + base_off + offset);
                }
            }
            float4 sum = part[0];
#pragma unroll
            for (int src = 1; src < 8; ++src) {
                if (src < splits) {
                    sum.x += part[src].x;
                    sum.y += part[src].y;
                    sum.z += part[src].z;
                    sum.w += part[src].w;
                }
            }
            const int grow = mb * TC_BM + r, gcol = nb * BN + q * 4;
            if (grow < p.m && gcol < p.n) {
                float *dst = p.c + static_cast<size_t>(grow) * p.n + gcol;
                if (vec && gcol + 3 < p.n) {
                    *reinterpret_cast<float4 *>(dst) = sum;
                } else {
                    const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
                    for (int e = 0; e < 4 && gcol + e < p.n; ++e)
                        dst[e] = vals[e];
                }
            }
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
