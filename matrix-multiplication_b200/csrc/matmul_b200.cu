// C-ABI of the B200 GEMM backend: context, validation, tensor maps, dispatch.
//
// Drop-in for the reference library src/matmul.cu (exports at :213-479): same
// five symbols, ABI version 3, the same 0/1 return convention with an
// "operation: detail" message in the caller's buffer, and the same rule that a
// failed cudaSetDevice leaves no sticky error behind (:280-283).  The kernels
// behind it are new: tcgen05 tensor-core GEMM (implementation 7) and an FFMA
// FP32 GEMM (implementation 8).  Declarations: include/b200_matmul.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <new>

#include "ffma_gemm.cuh"
#include "ffma_tma.cuh"
#include "pack.cuh"
#include "tc_gemm.cuh"
#include "tc2_gemm.cuh"
#include "tc_skinny.cuh"
#include "check.cuh"
#include "peer_push.cuh"
#include <cmath>

// Scratch for matmul_launch_noalloc: a fixed array in the module's device
// memory, so that entry point never allocates.  Every GPU that loads this
// library holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;   // 32 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

using namespace b200;

constexpr int kAbiVersion = 3;
constexpr int kImplTcgen05 = 7;
constexpr int kImplFfma = 8;
constexpr int kPrecFp32 = 0, kPrecTf32 = 1, kPrecFp16 = 2, kPrecBf16 = 3;
constexpr int kRasterGroupM = 16;
constexpr int kRasterGroupMPair = 8;
constexpr int kSkinnyMaxM = 64;        // m <= 64: swap-AB skinny kernel

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

struct Context {
    int device = 0;
    int major = 0;
    int minor = 0;
    // What the tensor-core launches may use: the device's SMs, or fewer after
    // matmul_set_sm_limit (the device_* fields keep the device's own values).
    int sm_count = 0;
    int max_pairs = 0;        // co-resident 2-CTA clusters of the pair kernel
    int max_split_ctas[4] = {}; // co-resident CTAs of the single-CTA kernel in (1,1,S) clusters, S = 1,2,4,8
    int device_sm_count = 0;
    int device_max_pairs = 0;
    int device_max_split_ctas[4] = {};
    int ffma_resident[2] = {}; // resident blocks per SM of each aligned FFMA tile
    EncodeTiledFn encode = nullptr;
    cudaMemPool_t pool = nullptr;
    // Device address of g_noalloc_scratch in this context's device, looked up by
    // the context's first matmul_launch_noalloc call with the device current (in
    // host code the symbol itself is a host-side stand-in, never a device
    // address).  Kept per context, so a context created after a device reset
    // looks it up again in the reloaded module.
    std::mutex noalloc_mutex;
    void *noalloc_scratch = nullptr;
    // Limit of the bounded waits that depend on another warp's progress
    // (matmul_set_wait_limit); 0 = the default.
    unsigned long long wait_limit_ns = 0;
};

unsigned long long wait_limit(const Context *ctx)
{
    return ctx->wait_limit_ns ? ctx->wait_limit_ns : kWaitLimitNs;
}

cudaError_t noalloc_scratch_address(Context *ctx, void **address)
{
    std::lock_guard<std::mutex> lock(ctx->noalloc_mutex);
    if (!ctx->noalloc_scratch) {
        void *ptr = nullptr;
        const cudaError_t st = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (st != cudaSuccess)
            return st;
        ctx->noalloc_scratch = ptr;
    }
    *address = ctx->noalloc_scratch;
    return cudaSuccess;
}

void clear_error(char *error, size_t error_size)
{
    if (error && error_size)
        error[0] = '\0';
}

int fail(char *error, size_t error_size, const char *operation, const char *detail)
{
    if (error && error_size)
        std::snprintf(error, error_size, "%s: %s", operation, detail);
    return 1;
}

int fail_cuda(char *error, size_t error_size, const char *operation, cudaError_t status)
{
    const char *detail = cudaGetErrorString(status);
    cudaGetLastError();
    return fail(error, error_size, operation, detail);
}

bool aligned16(const void *p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

int64_t round_up(int64_t x, int64_t to)
{
    return (x + to - 1) / to * to;
}

bool encode_2d(const Context *ctx, CUtensorMap *map, CUtensorMapDataType type, const void *base, uint64_t inner,
               uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B)
{
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = ctx->encode(map, type, 2, const_cast<void *>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Stream-ordered scratch: from the context's pool outside capture, as a graph
// allocation node inside capture.  Freed on the same stream after use.
cudaError_t scratch_alloc(Context *ctx, void **ptr, size_t bytes, cudaStream_t stream)
{
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    cudaError_t st = cudaStreamIsCapturing(stream, &capture);
    if (st != cudaSuccess)
        return st;
    if (capture == cudaStreamCaptureStatusActive || ctx->pool == nullptr)
        return cudaMallocAsync(ptr, bytes, stream);
    return cudaMallocFromPoolAsync(ptr, bytes, ctx->pool, stream);
}

// Launch with programmatic stream serialisation: the kernel may start while the
// previous kernel on the stream finishes; our kernels run their prologue and
// then wait (griddepcontrol.wait) before touching global memory.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args)
{
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

// launch_pdl with clusters of (1, 1, cluster_z) CTAs (cluster_z divides grid.z).
template <typename... Params, typename... Args>
cudaError_t launch_pdl_cluster_z(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, unsigned int cluster_z,
                                 cudaStream_t stream, Args &&...args)
{
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attributes[2]{};
    attributes[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[0].val.programmaticStreamSerializationAllowed = 1;
    attributes[1].id = cudaLaunchAttributeClusterDimension;
    attributes[1].val.clusterDim.x = 1;
    attributes[1].val.clusterDim.y = 1;
    attributes[1].val.clusterDim.z = cluster_z;
    config.attrs = attributes;
    config.numAttrs = cluster_z > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}


// Operands TMA cannot read in place (base not 16-byte aligned, or a row pitch
// that is not a multiple of 16 bytes), repacked into 16-byte aligned scratch in
// one launch (an operand with `direct` set is skipped).  TF32 operands are copied
// as FP32 words: the TMA loads round them.
template <typename T>
cudaError_t pack_operands(const Context *ctx, const void *a, bool a_direct, void *a_dst, int64_t m, int64_t k,
                          int64_t lda, const void *b, bool b_direct, void *b_dst, int64_t n, int64_t ldb,
                          cudaStream_t stream)
{
    if (a_direct && b_direct)
        return cudaSuccess;
    const PackJob<T> ja{static_cast<const T *>(a), static_cast<T *>(a_dst), a_direct ? 0 : m, k, lda};
    const PackJob<T> jb{static_cast<const T *>(b), static_cast<T *>(b_dst), b_direct ? 0 : k, n, ldb};
    const int64_t cap = 4LL * ctx->sm_count;
    auto blocks_for = [&](const PackJob<T> &j) {
        const int64_t blocks = (j.rows * j.ld + 255) / 256;
        return blocks < 1 ? int64_t{1} : blocks > cap ? cap : blocks;
    };
    const int64_t a_blocks = blocks_for(ja), b_blocks = blocks_for(jb);
    return launch_pdl(pack_pair_kernel<T>, dim3(static_cast<unsigned int>(a_blocks + b_blocks)), dim3(256), 0,
                      stream, ja, jb, static_cast<int>(a_blocks));
}

// tile_n selects the kernel: 0 = CTA pair with a 256 x 256 tile, 512 = CTA pair
// with a 256 x 512 tile, else the single-CTA kernel with a 128 x tile_n tile.
template <int FMT>
cudaError_t launch_tc_kernel(int tile_n, int splits, const CUtensorMap &ma, const CUtensorMap &mb,
                             const CUtensorMap &mc, const TcParams &params, int grid, cudaStream_t stream)
{
    const dim3 block(TC_THREADS);
    if (tile_n == 0)
        return launch_pdl(tc2_gemm_kernel<FMT, TC2_BN>, dim3(grid), block, Tc2Tile<TC2_BN>::kSmem, stream, ma, mb,
                          mc, params);
    if (tile_n == TC2W_BN)
        return launch_pdl(tc2_gemm_kernel<FMT, TC2W_BN>, dim3(grid), block, Tc2Tile<TC2W_BN>::kSmem, stream, ma,
                          mb, mc, params);
    // Split K: one tile per cluster of `splits` CTAs along z.
    const dim3 g = splits > 1 ? dim3(static_cast<unsigned int>(params.num_tiles), 1, static_cast<unsigned int>(splits))
                              : dim3(static_cast<unsigned int>(grid));
    const unsigned int cz = static_cast<unsigned int>(splits);
    if (tile_n == 256)
        return launch_pdl_cluster_z(tc_gemm_kernel<FMT, 256>, g, block, TcTile<256>::kSmem, cz, stream, ma, mb, mc,
                                    params);
    if (tile_n == 128)
        return launch_pdl_cluster_z(tc_gemm_kernel<FMT, 128>, g, block, TcTile<128>::kSmem, cz, stream, ma, mb, mc,
                                    params);
    if (params.a_box_rows <= 32)
        return launch_pdl_cluster_z(tc_gemm_kernel<FMT, 64, 32>, g, block, TcTile<64, 32>::kSmem, cz, stream, ma, mb,
                                    mc, params);
    return launch_pdl_cluster_z(tc_gemm_kernel<FMT, 64>, g, block, TcTile<64>::kSmem, cz, stream, ma, mb, mc,
                                params);
}

struct TcPlan {
    int tile_n;   // 0 = CTA pair (256 x 256), TC2W_BN = CTA pair (256 x 512), else the single-CTA tile width
    int splits;   // K splits (clusters of splits CTAs along z); single-CTA kernel only
};

// Launch plan of the tensor-core path: CTA pair or single-CTA tile width, and K
// splits.  Estimated cycles per option = fixed start-up + rounds x (K blocks x
// time per K block + epilogue) (+ the split reduction), where a K block costs the
// most of its MMA time (2 x tile width cycles), its operand bytes at 55 B/cycle
// into one SM, and all running CTAs' operand bytes at 8 KB/cycle out of L2; a
// split adds 1000 cycles plus its shared-memory exchange at 8 B/cycle, and the
// CTA pair 10000 cycles of start-up.  Fitted to measured B200 times of every
// option over square, long-K, skinny and ragged shapes in BF16 and TF32 (the
// chosen plan is within 3 % of the fastest on average).
double tc_plan_cycles(const Context *ctx, int m, int k, int n, int prec, int tile_n, int splits)
{
    constexpr double kStart = 2000.0, kEpilogue = 4000.0, kSmBytes = 55.0, kL2Bytes = 8000.0;
    const int64_t bk = prec == kPrecTf32 ? 32 : 64;
    const int64_t nkb = (static_cast<int64_t>(k) + bk - 1) / bk;
    int64_t tiles, rounds, active;
    double bytes_kb, mma;
    const bool pair = tile_n == 0 || tile_n == TC2W_BN;
    const int pair_n = tile_n == TC2W_BN ? TC2W_BN : TC2_BN;
    if (pair) {
        tiles = ((static_cast<int64_t>(m) + TC2_BM - 1) / TC2_BM) * ((static_cast<int64_t>(n) + pair_n - 1) / pair_n);
        rounds = (tiles + ctx->max_pairs - 1) / ctx->max_pairs;
        active = 2 * (tiles < ctx->max_pairs ? tiles : ctx->max_pairs);
        bytes_kb = static_cast<double>(TC2_HALF + pair_n / 2) * TC_ROW_BYTES;
        mma = 2.0 * pair_n;
    } else {
        tiles = ((static_cast<int64_t>(m) + TC_BM - 1) / TC_BM) * ((static_cast<int64_t>(n) + tile_n - 1) / tile_n);
        if (splits == 1) {
            rounds = (tiles + ctx->sm_count - 1) / ctx->sm_count;
            active = tiles < ctx->sm_count ? tiles : ctx->sm_count;
        } else {
            rounds = 1;
            active = tiles * splits;
        }
        bytes_kb = static_cast<double>(TC_BM + tile_n) * TC_ROW_BYTES;
        mma = 2.0 * tile_n;
    }
    const int64_t kpb = (nkb + splits - 1) / splits;
    double t_kb = mma;
    if (bytes_kb / kSmBytes > t_kb)
        t_kb = bytes_kb / kSmBytes;
    if (static_cast<double>(active) * bytes_kb / kL2Bytes > t_kb)
        t_kb = static_cast<double>(active) * bytes_kb / kL2Bytes;
    const double width = pair ? pair_n : tile_n;
    double cycles = kStart + static_cast<double>(rounds) * (static_cast<double>(kpb) * t_kb + kEpilogue * width / 256.0);
    if (pair)
        cycles += 10000.0;      // cluster launch, pair TMEM allocation and teardown
    if (splits > 1)
        cycles += 1000.0 + static_cast<double>(splits - 1) / splits * TC_BM * width * 4.0 / 8.0;
    return cycles;
}

TcPlan choose_tc_plan(const Context *ctx, int m, int k, int n, int prec)
{
    const int elem = prec == kPrecTf32 ? 4 : 2;
    const int64_t nkb = (static_cast<int64_t>(k) + TC_ROW_BYTES / elem - 1) / (TC_ROW_BYTES / elem);
    TcPlan best{64, 1};
    double best_cycles = 0.0;
    auto consider = [&](int tile_n, int splits) {
        const double cycles = tc_plan_cycles(ctx, m, k, n, prec, tile_n, splits);
        if (best_cycles == 0.0 || cycles < best_cycles) {
            best = {tile_n, splits};
            best_cycles = cycles;
        }
    };
    if (m > TC_BM && ctx->max_pairs > 0) {
        consider(0, 1);
        if (n > TC2_BN)
            consider(TC2W_BN, 1);
    }
    for (int tile_n : {256, 128, 64}) {
        const int64_t tiles =
            ((static_cast<int64_t>(m) + TC_BM - 1) / TC_BM) * ((static_cast<int64_t>(n) + tile_n - 1) / tile_n);
        for (int i = 0; i < 4; ++i) {
            const int splits = 1 << i;
            if (splits > 1) {
                // One wave of whole clusters, every split with K blocks of its own, and
                // room for the exchanged partial tiles (S <= 4 for 256-wide tiles).
                const int64_t kpb = (nkb + splits - 1) / splits;
                if ((tile_n == 256 && splits > 4) || tiles * splits > ctx->max_split_ctas[i] ||
                    (splits - 1) * kpb >= nkb)
                    continue;
            }
            consider(tile_n, splits);
        }
    }
    return best;
}

// K splits of the skinny kernel: the most (1, 2, 4 or 8) whose clusters all fit
// on the device at once with at least four K blocks per split.  The kernel is
// HBM-bound on B, so more SMs streaming it is what counts.
int skinny_splits(const Context *ctx, int n, int total_k_blocks)
{
    const int64_t tiles = (n + SK_BM - 1) / SK_BM;
    int best = 1;
    for (int i = 1; i < 4; ++i) {
        const int splits = 1 << i;
        const int64_t kpb = (total_k_blocks + splits - 1) / splits;
        if (tiles * splits <= ctx->max_split_ctas[i] && kpb >= 4 && (splits - 1) * kpb < total_k_blocks)
            best = splits;
    }
    return best;
}

template <int FMT, int NP>
cudaError_t launch_skinny_kernel(const CUtensorMap &mbt, const CUtensorMap &mat, const SkParams &params, dim3 grid,
                                 cudaStream_t stream)
{
    return launch_pdl_cluster_z(tc_skinny_kernel<FMT, NP>, grid, dim3(TC_THREADS), SkTile<NP>::kSmem, grid.z, stream,
                                mbt, mat, params);
}

template <int FMT>
cudaError_t launch_skinny_np(int np, const CUtensorMap &mbt, const CUtensorMap &mat, const SkParams &params,
                             dim3 grid, cudaStream_t stream)
{
    if (np == 16)
        return launch_skinny_kernel<FMT, 16>(mbt, mat, params, grid, stream);
    if (np == 32)
        return launch_skinny_kernel<FMT, 32>(mbt, mat, params, grid, stream);
    return launch_skinny_kernel<FMT, 64>(mbt, mat, params, grid, stream);
}

// m <= 64: C^T = B^T A^T with N on the MMA's 128-row side (tc_skinny.cuh).  The
// operands are already in TMA-ready form (a_op: m x lda; b_op: k x ldb).
int launch_skinny(Context *ctx, int prec, const void *a_op, int64_t lda, const void *b_op, int64_t ldb,
                  float *c, int m, int k, int n, cudaStream_t stream, char *error, size_t error_size)
{
    const int elem = prec == kPrecTf32 ? 4 : 2;
    const uint32_t bk = TC_ROW_BYTES / elem;
    const int np = m <= 16 ? 16 : m <= 32 ? 32 : 64;
    const CUtensorMapDataType type = prec == kPrecTf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32
                                     : prec == kPrecBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    alignas(64) CUtensorMap map_bt, map_at;
    const CUtensorMapSwizzle b_swizzle =
        prec == kPrecTf32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    bool ok = encode_2d(ctx, &map_bt, type, b_op, static_cast<uint64_t>(n), static_cast<uint64_t>(k),
                        static_cast<uint64_t>(ldb) * elem, TC_ROW_BYTES / elem, SK_B_ROWS, b_swizzle);
    ok = ok && encode_2d(ctx, &map_at, type, a_op, static_cast<uint64_t>(k), static_cast<uint64_t>(m),
                         static_cast<uint64_t>(lda) * elem, bk, static_cast<uint32_t>(np));
    if (!ok) {
        cudaGetLastError();
        return fail(error, error_size, "matmul_launch", "cuTensorMapEncodeTiled rejected an operand");
    }
    SkParams params{};
    params.m = m;
    params.n = n;
    params.k = k;
    params.num_n_tiles = (n + SK_BM - 1) / SK_BM;
    params.total_k_blocks = static_cast<int>((static_cast<int64_t>(k) + bk - 1) / bk);
    const int splits = skinny_splits(ctx, n, params.total_k_blocks);
    params.num_k_blocks = (params.total_k_blocks + splits - 1) / splits;
    params.c = c;
    params.wait_limit_ns = wait_limit(ctx);
    // Split K: one 128-column slab per cluster of `splits` CTAs along z.
    const dim3 grid = splits > 1 ? dim3(static_cast<unsigned int>(params.num_n_tiles), 1,
                                        static_cast<unsigned int>(splits))
                                 : dim3(static_cast<unsigned int>(params.num_n_tiles < ctx->sm_count
                                                                      ? params.num_n_tiles
                                                                      : ctx->sm_count));
    cudaError_t st;
    if (prec == kPrecTf32)
        st = launch_skinny_np<kFmtTF32>(np, map_bt, map_at, params, grid, stream);
    else if (prec == kPrecBf16)
        st = launch_skinny_np<kFmtBF16>(np, map_bt, map_at, params, grid, stream);
    else
        st = launch_skinny_np<kFmtF16>(np, map_bt, map_at, params, grid, stream);
    if (st != cudaSuccess)
        return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
    return 0;
}

bool tf32_on_ffma(int m, int k, int n);
int launch_ffma_tf32(const Context *ctx, const float *a, const float *b, float *c, int m, int k, int n,
                     cudaStream_t stream, char *error, size_t error_size);

int launch_tcgen05(Context *ctx, int prec, const void *a, const void *b, float *c, int m, int k, int n,
                   cudaStream_t stream, char *error, size_t error_size, void *fixed_scratch = nullptr,
                   size_t fixed_scratch_bytes = 0)
{
    if (prec == kPrecTf32 && tf32_on_ffma(m, k, n))
        return launch_ffma_tf32(ctx, static_cast<const float *>(a), static_cast<const float *>(b), c, m, k, n,
                                stream, error, error_size);
    const int elem = prec == kPrecTf32 ? 4 : 2;
    const int64_t align_elems = 16 / elem;
    // TMA needs 16-byte aligned bases and row pitches; operands without them are
    // repacked.  TF32 operands are read as FP32 words through TFLOAT32 tensor maps,
    // whose loads round each word to TF32 (nearest even, the reference's
    // round_tf32_even), so TF32 needs no pass of its own.
    const bool a_direct = aligned16(a) && (static_cast<int64_t>(k) * elem) % 16 == 0;
    const bool b_direct = aligned16(b) && (static_cast<int64_t>(n) * elem) % 16 == 0;
    const int64_t lda = a_direct ? k : round_up(k, align_elems);
    const int64_t ldb = b_direct ? n : round_up(n, align_elems);
    const size_t a_bytes = a_direct ? 0 : static_cast<size_t>(round_up(static_cast<int64_t>(m) * lda * elem, 256));
    const size_t b_bytes = b_direct ? 0 : static_cast<size_t>(round_up(static_cast<int64_t>(k) * ldb * elem, 256));

    void *scratch = nullptr;
    if (a_bytes + b_bytes && fixed_scratch) {
        if (a_bytes + b_bytes > fixed_scratch_bytes) {
            char detail[200];
            std::snprintf(detail, sizeof(detail),
                          "this problem needs %zu bytes of scratch, more than the fixed %zu-byte array; "
                          "use matmul_launch",
                          a_bytes + b_bytes, fixed_scratch_bytes);
            return fail(error, error_size, "matmul_launch_noalloc", detail);
        }
        scratch = fixed_scratch;
    } else if (a_bytes + b_bytes) {
        const cudaError_t st = scratch_alloc(ctx, &scratch, a_bytes + b_bytes, stream);
        if (st != cudaSuccess)
            return fail_cuda(error, error_size, "matmul_launch: scratch allocation", st);
    }
    // Only scratch taken from the stream-ordered pool is handed back.
    void *pooled = fixed_scratch ? nullptr : scratch;
    const void *a_op = a_direct ? a : scratch;
    const void *b_op = b_direct ? b : static_cast<uint8_t *>(scratch) + a_bytes;
    {
        const cudaError_t st =
            prec == kPrecTf32
                ? pack_operands<float>(ctx, a, a_direct, const_cast<void *>(a_op), m, k, lda, b, b_direct,
                                       const_cast<void *>(b_op), n, ldb, stream)
            : prec == kPrecBf16
                ? pack_operands<__nv_bfloat16>(ctx, a, a_direct, const_cast<void *>(a_op), m, k, lda, b, b_direct,
                                               const_cast<void *>(b_op), n, ldb, stream)
                : pack_operands<__half>(ctx, a, a_direct, const_cast<void *>(a_op), m, k, lda, b, b_direct,
                                        const_cast<void *>(b_op), n, ldb, stream);
        if (st != cudaSuccess) {
            if (pooled)
                cudaFreeAsync(pooled, stream);
            return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
        }
    }

    if (m <= kSkinnyMaxM) {
        const int rc = launch_skinny(ctx, prec, a_op, lda, b_op, ldb, c, m, k, n, stream, error, error_size);
        if (pooled)
            cudaFreeAsync(pooled, stream);
        return rc;
    }

    const TcPlan plan = choose_tc_plan(ctx, m, k, n, prec);
    const int kernel_n = plan.tile_n;
    const bool pair = kernel_n == 0 || kernel_n == TC2W_BN;
    const int tile_m = pair ? TC2_BM : TC_BM;
    const int tile_n = kernel_n == 0 ? TC2_BN : kernel_n;
    const CUtensorMapDataType type = prec == kPrecTf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32
                                     : prec == kPrecBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t bk = TC_ROW_BYTES / elem;
    alignas(64) CUtensorMap map_a, map_b, map_c;
    std::memset(&map_c, 0, sizeof(map_c));
    // Skinny problems (m < 128) fetch only the rows that exist.
    const int a_box_rows = pair || m >= TC_BM ? TC_BM : static_cast<int>(round_up(m, 16));
    bool ok = encode_2d(ctx, &map_a, type, a_op, static_cast<uint64_t>(k), static_cast<uint64_t>(m),
                        static_cast<uint64_t>(lda) * elem, bk, static_cast<uint32_t>(a_box_rows));
    ok = ok && encode_2d(ctx, &map_b, type, b_op, static_cast<uint64_t>(n), static_cast<uint64_t>(k),
                         static_cast<uint64_t>(ldb) * elem, TC_ROW_BYTES / elem, bk,
                         prec == kPrecTf32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
    const bool c_direct = !(aligned16(c) && n % 4 == 0);
    if (ok && !c_direct)
        ok = encode_2d(ctx, &map_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, c, static_cast<uint64_t>(n),
                       static_cast<uint64_t>(m), static_cast<uint64_t>(n) * 4, 32, TC_BM);
    if (!ok) {
        if (pooled)
            cudaFreeAsync(pooled, stream);
        cudaGetLastError();
        return fail(error, error_size, "matmul_launch", "cuTensorMapEncodeTiled rejected an operand");
    }

    TcParams params{};
    params.m = m;
    params.n = n;
    params.k = k;
    params.num_m_blocks = (m + tile_m - 1) / tile_m;
    params.num_n_blocks = (n + tile_n - 1) / tile_n;
    params.num_k_blocks = static_cast<int>((static_cast<int64_t>(k) + bk - 1) / bk);
    const int64_t tiles = static_cast<int64_t>(params.num_m_blocks) * params.num_n_blocks;
    if (tiles > 0x7fffffff) {
        if (pooled)
            cudaFreeAsync(pooled, stream);
        return fail(error, error_size, "matmul_launch", "too many output tiles");
    }
    params.num_tiles = static_cast<int>(tiles);
    // 8 pair blocks (2048 rows) or 16 single blocks per raster group: about as
    // many A row blocks as B column blocks in flight across the 148 SMs.
    params.group_m = pair ? kRasterGroupMPair : kRasterGroupM;
    params.c = c;
    params.c_direct = c_direct ? 1 : 0;
    params.a_box_rows = a_box_rows;
    params.wait_limit_ns = wait_limit(ctx);
    const int units = pair ? ctx->max_pairs : ctx->sm_count;
    const int grid = static_cast<int>(tiles < units ? tiles : units) * (pair ? 2 : 1);

    cudaError_t st;
    if (prec == kPrecTf32)
        st = launch_tc_kernel<kFmtTF32>(kernel_n, plan.splits, map_a, map_b, map_c, params, grid, stream);
    else if (prec == kPrecBf16)
        st = launch_tc_kernel<kFmtBF16>(kernel_n, plan.splits, map_a, map_b, map_c, params, grid, stream);
    else
        st = launch_tc_kernel<kFmtF16>(kernel_n, plan.splits, map_a, map_b, map_c, params, grid, stream);
    if (pooled)
        cudaFreeAsync(pooled, stream);
    if (st != cudaSuccess)
        return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
    return 0;
}


// Launch plan of the FFMA kernel: output tile and K split.  The busiest SM's
// time is estimated as (its blocks) x (tile area) x (16-deep K steps per split) /
// efficiency, where efficiency falls when fewer than about 17 warps are resident
// (0.3 + warps / 24) and the 32 x 32 tile's 4 x 4 micro-tile is 40 % less
// efficient than the 8 x 8 one; plus, per wave of resident blocks, a pipeline
// fill and epilogue worth two K steps and, when split, the cluster exchange worth
// eight.  Fitted to measured B200 times of every tile and split over square sizes
// 64-4096, skinny / long-K and ragged (unaligned, short-K) shapes: the chosen
// plan is within 2.4 % of the fastest on average, 14 % at worst.  128 x 64 and
// 64 x 64 tiles were measured too and never won by enough to keep.
struct FfmaTileOption {
    int bm, bn, warps, bk;
    double efficiency;
};
constexpr FfmaTileOption kFfmaTiles[] = {{128, 128, 8, FaTile<128, 128, 8, 8>::kBK, 1.0},
                                         {32, 32, 2, FaTile<32, 32, 4, 4>::kBK, 0.6}};
constexpr int kFfmaTileCount = sizeof(kFfmaTiles) / sizeof(kFfmaTiles[0]);
constexpr int kFfmaMaxSplits = 8;                       // portable cluster size

struct FfmaPlan {
    int tile;
    int splits;
};

FfmaPlan choose_ffma_plan(int m, int k, int n, int sm_count, const int *resident, unsigned tiles_allowed = 3u)
{
    FfmaPlan best{0, 1};
    double best_cost = 0.0;
    // Work in 16-deep K units; a split never has fewer K tiles of its own depth than one.
    const int64_t total_kt = (static_cast<int64_t>(k) + FA_MODEL_BK - 1) / FA_MODEL_BK;
    bool have = false;
    for (int t = 0; t < kFfmaTileCount; ++t) {
        if (!((tiles_allowed >> t) & 1u))
            continue;
        const FfmaTileOption &o = kFfmaTiles[t];
        const int64_t tile_kt = (static_cast<int64_t>(k) + o.bk - 1) / o.bk;
        const int64_t tiles = ((static_cast<int64_t>(m) + o.bm - 1) / o.bm) *
                              ((static_cast<int64_t>(n) + o.bn - 1) / o.bn);
        const int64_t slots = resident[t] > 0 ? resident[t] : 1;
        for (int splits = 1; splits <= kFfmaMaxSplits && splits <= tile_kt; splits *= 2) {
            const int64_t per_sm = (tiles * splits + sm_count - 1) / sm_count;
            const int64_t concurrent = per_sm < slots ? per_sm : slots;
            const int64_t waves = (per_sm + slots - 1) / slots;
            const int64_t kt = (total_kt + splits - 1) / splits;
            const double occupancy = 0.3 + static_cast<double>(concurrent * o.warps) / 24.0;
            const double efficiency = o.efficiency * (occupancy < 1.0 ? occupancy : 1.0);
            const double area = static_cast<double>(o.bm) * o.bn;
            const double cost = static_cast<double>(per_sm) * area * static_cast<double>(kt) / efficiency +
                                (splits > 1 ? 8.0 : 2.0) * static_cast<double>(waves * concurrent) * area;
            if (!have || cost < best_cost * 0.999) {
                best = {t, splits};
                best_cost = cost;
                have = true;
            }
        }
    }
    return best;
}

template <int BM, int BN, int RM, int RN, bool VEC_AB, bool TF32_ROUND = false>
cudaError_t launch_ffma_async(const float *a, const float *b, float *c, int m, int k, int n, int splits, bool vec_c,
                              cudaStream_t stream)
{
    using T = FaTile<BM, BN, RM, RN>;
    const int64_t gx = (static_cast<int64_t>(n) + BN - 1) / BN;
    const int64_t gy = (static_cast<int64_t>(m) + BM - 1) / BM;
    const dim3 grid(static_cast<unsigned int>(gx < 65535 ? gx : 65535),
                    static_cast<unsigned int>(gy < 65535 ? gy : 65535), static_cast<unsigned int>(splits));
    if (vec_c)
        return launch_pdl_cluster_z(ffma_gemm_async_kernel<BM, BN, RM, RN, VEC_AB, true, TF32_ROUND>, grid,
                                    dim3(T::kThreads), T::kSmemBytes, splits, stream, a, b, c, m, n, k);
    return launch_pdl_cluster_z(ffma_gemm_async_kernel<BM, BN, RM, RN, VEC_AB, false, TF32_ROUND>, grid,
                                dim3(T::kThreads), T::kSmemBytes, splits, stream, a, b, c, m, n, k);
}

template <bool VEC_AB>
cudaError_t launch_ffma_plan(const FfmaPlan &plan, const float *a, const float *b, float *c, int m, int k, int n,
                             bool vec_c, cudaStream_t stream)
{
    if (plan.tile == 0)
        return launch_ffma_async<128, 128, 8, 8, VEC_AB>(a, b, c, m, k, n, plan.splits, vec_c, stream);
    return launch_ffma_async<32, 32, 4, 4, VEC_AB>(a, b, c, m, k, n, plan.splits, vec_c, stream);
}

// TF32 problems this small run on the FFMA kernel with each K tile rounded to
// TF32 in shared memory (the TF32 products are exact in FP32): below about 320^3 the
// tensor-core path's start-up costs more than the FMAs
// (measured: 64^3-256^3 TF32 at 5.4-7.8 us on the tensor cores, 2.9-4.4 us here).
bool tf32_on_ffma(int m, int k, int n)
{
    return static_cast<int64_t>(m) * k * n <= (int64_t{1} << 25);
}

// The TF32 form of the FFMA launch: 32 x 32 tiles only.
int launch_ffma_tf32(const Context *ctx, const float *a, const float *b, float *c, int m, int k, int n,
                     cudaStream_t stream, char *error, size_t error_size)
{
    const bool vec_ab = aligned16(a) && k % 4 == 0 && aligned16(b) && n % 4 == 0;
    const bool vec_c = aligned16(c) && n % 4 == 0;
    const FfmaPlan plan = choose_ffma_plan(m, k, n, ctx->sm_count, ctx->ffma_resident, 2u);
    const cudaError_t st = vec_ab ? launch_ffma_async<32, 32, 4, 4, true, true>(a, b, c, m, k, n, plan.splits, vec_c, stream)
                                  : launch_ffma_async<32, 32, 4, 4, false, true>(a, b, c, m, k, n, plan.splits, vec_c,
                                                                                 stream);
    if (st != cudaSuccess)
        return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
    return 0;
}

// The 128 x 128 FFMA tile with TMA-staged operands (ffma_tma.cuh); needs 16-byte
// aligned operands and row pitches, which the caller has checked.
cudaError_t launch_ffma_tma(const Context *ctx, const float *a, const float *b, float *c, int m, int k, int n,
                            int splits, bool vec_c, cudaStream_t stream, bool &encoded)
{
    alignas(64) CUtensorMap map_a, map_b;
    encoded = encode_2d(ctx, &map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a, static_cast<uint64_t>(k),
                        static_cast<uint64_t>(m), static_cast<uint64_t>(k) * 4, FT_BK, FT_BM) &&
              encode_2d(ctx, &map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, b, static_cast<uint64_t>(n),
                        static_cast<uint64_t>(k), static_cast<uint64_t>(n) * 4, 32, FT_BK);
    if (!encoded)
        return cudaSuccess;
    FtParams params{};
    params.m = m;
    params.n = n;
    params.k = k;
    params.c = c;
    params.wait_limit_ns = wait_limit(ctx);
    const int64_t gx = (static_cast<int64_t>(n) + FT_BN - 1) / FT_BN;
    const int64_t gy = (static_cast<int64_t>(m) + FT_BM - 1) / FT_BM;
    const dim3 grid(static_cast<unsigned int>(gx < 65535 ? gx : 65535),
                    static_cast<unsigned int>(gy < 65535 ? gy : 65535), static_cast<unsigned int>(splits));
    if (vec_c)
        return launch_pdl_cluster_z(ffma_tma_kernel<true>, grid, dim3(FT_THREADS), FT_SMEM, splits, stream, map_a,
                                    map_b, params);
    return launch_pdl_cluster_z(ffma_tma_kernel<false>, grid, dim3(FT_THREADS), FT_SMEM, splits, stream, map_a,
                                map_b, params);
}

int launch_ffma(const Context *ctx, const float *a, const float *b, float *c, int m, int k, int n,
                cudaStream_t stream, char *error, size_t error_size)
{
    // 16-byte aligned operands: the 128 x 128 tile is staged by TMA, the 32 x 32
    // tile by 16-byte cp.async; otherwise 4-byte cp.async copies.
    const bool vec_ab = aligned16(a) && k % 4 == 0 && aligned16(b) && n % 4 == 0;
    const bool vec_c = aligned16(c) && n % 4 == 0;
    const FfmaPlan plan = choose_ffma_plan(m, k, n, ctx->sm_count, ctx->ffma_resident);
    if (vec_ab && plan.tile == 0) {
        bool encoded = false;
        const cudaError_t st = launch_ffma_tma(ctx, a, b, c, m, k, n, plan.splits, vec_c, stream, encoded);
        if (!encoded) {
            cudaGetLastError();
            return fail(error, error_size, "matmul_launch", "cuTensorMapEncodeTiled rejected an operand");
        }
        if (st != cudaSuccess)
            return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
        return 0;
    }
    const cudaError_t st = vec_ab ? launch_ffma_plan<true>(plan, a, b, c, m, k, n, vec_c, stream)
                                  : launch_ffma_plan<false>(plan, a, b, c, m, k, n, vec_c, stream);
    if (st != cudaSuccess)
        return fail(error, error_size, "kernel launch", cudaGetErrorString(st));
    return 0;
}

const char *kPrecisionNames[] = {"fp32", "tf32", "fp16", "bf16"};

bool supported(int implementation, int precision)
{
    if (implementation == kImplTcgen05)
        return precision == kPrecTf32 || precision == kPrecFp16 || precision == kPrecBf16;
    if (implementation == kImplFfma)
        return precision == kPrecFp32;
    return false;
}

int check_ids(int implementation, int precision, const char *op, char *error, size_t error_size)
{
    if (precision < 0 || precision > 3)
        return fail(error, error_size, op, "unknown precision");
    if (implementation >= 0 && implementation <= 6)
        return fail(error, error_size, op,
                    "implementations 0-6 (the sm_80 reference kernels and cuBLAS) are not part of this "
                    "library; use 7 (tcgen05) or 8 (ffma)");
    if (implementation != kImplTcgen05 && implementation != kImplFfma)
        return fail(error, error_size, op, "unknown implementation");
    if (!supported(implementation, precision))
        return fail(error, error_size, op, "unsupported implementation and precision");
    return 0;
}

} // namespace

extern "C" int matmul_abi_version()
{
    return kAbiVersion;
}

extern "C" int matmul_kernel_info(int implementation, int precision, char *json, size_t json_size, char *error,
                                  size_t error_size)
{
    clear_error(error, error_size);
    if (!json || !json_size)
        return fail(error, error_size, "matmul_kernel_info", "JSON buffer is null or empty");
    json[0] = '\0';
    if (check_ids(implementation, precision, "matmul_kernel_info", error, error_size))
        return 1;
    int written;
    if (implementation == kImplTcgen05) {
        const int elem = precision == kPrecTf32 ? 4 : 2;
        written = std::snprintf(
            json, json_size,
            "{\"implementation\":\"tcgen05\",\"precision\":\"%s\",\"tile_m\":%d,\"tile_n\":%d,"
            "\"tile_k\":%d,\"threads\":%d,\"warp_tile_m\":%d,\"warp_tile_n\":%d,\"microtile_m\":%d,"
            "\"microtile_n\":%d,\"buffering\":%d,\"load_method\":\"tma_sw128\",\"tensor_cores\":true,"
            "\"mma\":\"tcgen05.mma.cta_group::2.kind::%s\",\"mma_shape\":[%d,%d,%d],\"cluster\":[2,1,1],"
            "\"accumulator\":\"tmem_fp32\",\"tmem_columns\":%u,\"accumulator_buffers\":2,"
            "\"warp_roles\":{\"tma\":1,\"mma\":1,\"epilogue\":4},\"schedule\":\"persistent\","
            "\"raster_group_m\":%d,\"epilogue\":\"tmem_ld_smem_tma_store\",\"input_rounding\":\"%s\","
            "\"b_operand\":\"%s\",\"plan\":\"cost_model\",\"single_cta_kernel\":{\"tile_m\":%d,"
            "\"tile_n\":[256,128,64],\"buffering\":[%d,%d,%d],\"raster_group_m\":%d,"
            "\"split_k\":\"cluster_1x1xS_bulk_copy\",\"max_splits\":8},"
            "\"pair_wide_kernel\":{\"tile_n\":%d,\"buffering\":%d,\"accumulator\":\"one, freed in column halves\"},\"skinny_kernel\":{\"when\":\"m<=64\",\"tile_n\":%d,\"max_splits\":8},"
            "\"small_tf32\":\"ffma_tf32_rne when m*k*n<=2^25\"}",
            kPrecisionNames[precision], TC2_BM, TC2_BN, TC_ROW_BYTES / elem, TC_THREADS, TC2_HALF, TC2_BN, TC2_HALF,
            TC2_BN, TC2_STAGES, precision == kPrecTf32 ? "tf32" : "f16", TC2_BM, TC2_BN, 32 / elem,
            TC_TMEM_COLUMNS, kRasterGroupMPair, precision == kPrecTf32 ? "rne_by_tma_tfloat32_loads" : "none",
            precision == kPrecTf32 ? "mn_major_tma_sw128_atom32B" : "mn_major_tma_sw128", TC_BM, TcTile<256>::kStages,
            TcTile<128>::kStages, TcTile<64>::kStages, kRasterGroupM, TC2W_BN, Tc2Tile<TC2W_BN>::kStages, SK_BM);
    } else {
        written = std::snprintf(
            json, json_size,
            "{\"implementation\":\"ffma\",\"precision\":\"fp32\",\"tile_m\":%d,\"tile_n\":%d,"
            "\"tile_k\":%d,\"threads\":%d,\"warp_tile_m\":%d,\"warp_tile_n\":%d,\"microtile_m\":8,"
            "\"microtile_n\":8,\"buffering\":%d,\"load_method\":\"tma_sw128 when A and B rows are 16-byte "
            "aligned, else cp_async_zero_fill\","
            "\"copy_bytes\":\"TMA boxes (aligned 128 x 128 tile), 16-byte cp.async (aligned 32 x 32 tile), else 4\","
            "\"tensor_cores\":false,\"fma\":\"ffma2_rn_packed_fp32x2\",\"blocks_per_sm\":2,"
            "\"small_tiles\":[[32,32,4,4]],\"split_k\":\"cluster_1x1xS_dsmem_reduce\","
            "\"max_splits\":%d,\"plan_choice\":\"cost_model_busiest_sm\"}",
            FF_BM, FF_BN, FaTile<128, 128, 8, 8>::kBK, FF_THREADS, 16, 128, FaTile<128, 128, 8, 8>::kStages,
            kFfmaMaxSplits);
    }
    if (written < 0 || static_cast<size_t>(written) >= json_size) {
        json[0] = '\0';
        return fail(error, error_size, "matmul_kernel_info", "JSON buffer too small");
    }
    return 0;
}

extern "C" void *matmul_create(int device, char *error, size_t error_size)
{
    clear_error(error, error_size);
    cudaError_t st = cudaSetDevice(device);
    if (st != cudaSuccess) {
        fail_cuda(error, error_size, "cudaSetDevice", st);
        return nullptr;
    }
    int major = 0, minor = 0, sms = 0;
    st = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (st == cudaSuccess)
        st = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (st == cudaSuccess)
        st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (st != cudaSuccess) {
        fail_cuda(error, error_size, "cudaDeviceGetAttribute", st);
        return nullptr;
    }
    if (major != 10 || minor != 0) {
        char detail[160];
        std::snprintf(detail, sizeof(detail),
                      "device %d has compute capability %d.%d; this library contains sm_100a code only", device,
                      major, minor);
        fail(error, error_size, "matmul_create", detail);
        return nullptr;
    }

    Context *ctx = new (std::nothrow) Context{};
    if (!ctx) {
        fail(error, error_size, "matmul_create", "could not allocate context");
        return nullptr;
    }
    ctx->device = device;
    ctx->major = major;
    ctx->minor = minor;
    ctx->sm_count = sms;

    void *fn = nullptr;
    cudaDriverEntryPointQueryResult query{};
    st = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &query);
    if (st != cudaSuccess || query != cudaDriverEntryPointSuccess || !fn) {
        delete ctx;
        if (st != cudaSuccess)
            fail_cuda(error, error_size, "cudaGetDriverEntryPoint", st);
        else
            fail(error, error_size, "cudaGetDriverEntryPoint", "cuTensorMapEncodeTiled not found");
        return nullptr;
    }
    ctx->encode = reinterpret_cast<EncodeTiledFn>(fn);

    const std::pair<const void *, int> tc_kernels[] = {
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtF16, 256>), TcTile<256>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtBF16, 256>), TcTile<256>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtTF32, 256>), TcTile<256>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtF16, 128>), TcTile<128>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtBF16, 128>), TcTile<128>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtTF32, 128>), TcTile<128>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtF16, 64>), TcTile<64>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtBF16, 64>), TcTile<64>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtTF32, 64>), TcTile<64>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtF16, 64, 32>), TcTile<64, 32>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtBF16, 64, 32>), TcTile<64, 32>::kSmem},
        {reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtTF32, 64, 32>), TcTile<64, 32>::kSmem}};
    for (const auto &kernel : tc_kernels) {
        st = cudaFuncSetAttribute(kernel.first, cudaFuncAttributeMaxDynamicSharedMemorySize, kernel.second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
#define B200_FFMA_KERNEL(BM, BN, RM, RN, VAB, VC)                                                              \
    {reinterpret_cast<const void *>(&ffma_gemm_async_kernel<BM, BN, RM, RN, VAB, VC>),                          \
     FaTile<BM, BN, RM, RN>::kSmemBytes}
    // Per tile: the (vector A/B, vector C) variant first, whose occupancy the plan uses.
    const std::pair<const void *, int> ffma_kernels[] = {
        B200_FFMA_KERNEL(128, 128, 8, 8, true, true),  B200_FFMA_KERNEL(128, 128, 8, 8, true, false),
        B200_FFMA_KERNEL(128, 128, 8, 8, false, true), B200_FFMA_KERNEL(128, 128, 8, 8, false, false),
        B200_FFMA_KERNEL(32, 32, 4, 4, true, true),    B200_FFMA_KERNEL(32, 32, 4, 4, true, false),
        B200_FFMA_KERNEL(32, 32, 4, 4, false, true),   B200_FFMA_KERNEL(32, 32, 4, 4, false, false)};
    const std::pair<const void *, int> ffma_tf32_kernels[] = {
        {reinterpret_cast<const void *>(&ffma_gemm_async_kernel<32, 32, 4, 4, true, true, true>),
         FaTile<32, 32, 4, 4>::kSmemBytes},
        {reinterpret_cast<const void *>(&ffma_gemm_async_kernel<32, 32, 4, 4, true, false, true>),
         FaTile<32, 32, 4, 4>::kSmemBytes},
        {reinterpret_cast<const void *>(&ffma_gemm_async_kernel<32, 32, 4, 4, false, true, true>),
         FaTile<32, 32, 4, 4>::kSmemBytes},
        {reinterpret_cast<const void *>(&ffma_gemm_async_kernel<32, 32, 4, 4, false, false, true>),
         FaTile<32, 32, 4, 4>::kSmemBytes}};
    for (const auto &kernel : ffma_tf32_kernels) {
        st = cudaFuncSetAttribute(kernel.first, cudaFuncAttributeMaxDynamicSharedMemorySize, kernel.second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
#undef B200_FFMA_KERNEL
    for (const void *kernel : {reinterpret_cast<const void *>(&ffma_tma_kernel<true>),
                               reinterpret_cast<const void *>(&ffma_tma_kernel<false>)}) {
        st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FT_SMEM);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
    for (const auto &kernel : ffma_kernels) {
        st = cudaFuncSetAttribute(kernel.first, cudaFuncAttributeMaxDynamicSharedMemorySize, kernel.second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
    static_assert(sizeof(ffma_kernels) / sizeof(ffma_kernels[0]) == 4 * kFfmaTileCount, "four variants per tile");
    for (int t = 0; t < kFfmaTileCount; ++t) {
        const int threads = kFfmaTiles[t].warps * 32;
        st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctx->ffma_resident[t], ffma_kernels[4 * t].first,
                                                           threads, ffma_kernels[4 * t].second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaOccupancyMaxActiveBlocksPerMultiprocessor", st);
            return nullptr;
        }
    }
    const std::pair<const void *, int> skinny_kernels[] = {
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtF16, 16>), SkTile<16>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtBF16, 16>), SkTile<16>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtTF32, 16>), SkTile<16>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtF16, 32>), SkTile<32>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtBF16, 32>), SkTile<32>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtTF32, 32>), SkTile<32>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtF16, 64>), SkTile<64>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtBF16, 64>), SkTile<64>::kSmem},
        {reinterpret_cast<const void *>(&tc_skinny_kernel<kFmtTF32, 64>), SkTile<64>::kSmem}};
    for (const auto &kernel : skinny_kernels) {
        st = cudaFuncSetAttribute(kernel.first, cudaFuncAttributeMaxDynamicSharedMemorySize, kernel.second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
    const std::pair<const void *, int> tc2_kernels[] = {
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtF16, TC2_BN>), Tc2Tile<TC2_BN>::kSmem},
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtBF16, TC2_BN>), Tc2Tile<TC2_BN>::kSmem},
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtTF32, TC2_BN>), Tc2Tile<TC2_BN>::kSmem},
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtF16, TC2W_BN>), Tc2Tile<TC2W_BN>::kSmem},
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtBF16, TC2W_BN>), Tc2Tile<TC2W_BN>::kSmem},
        {reinterpret_cast<const void *>(&tc2_gemm_kernel<kFmtTF32, TC2W_BN>), Tc2Tile<TC2W_BN>::kSmem}};
    for (const auto &kernel : tc2_kernels) {
        st = cudaFuncSetAttribute(kernel.first, cudaFuncAttributeMaxDynamicSharedMemorySize, kernel.second);
        if (st != cudaSuccess) {
            delete ctx;
            fail_cuda(error, error_size, "cudaFuncSetAttribute", st);
            return nullptr;
        }
    }
    // How many 2-CTA clusters of the pair kernels (both widths) fit on the device at once.
    ctx->max_pairs = -1;
    for (int i : {1, 4}) {
        cudaLaunchConfig_t config{};
        config.gridDim = dim3(2 * (sms / 2), 1, 1);
        config.blockDim = dim3(TC_THREADS, 1, 1);
        config.dynamicSmemBytes = static_cast<size_t>(tc2_kernels[i].second);
        cudaLaunchAttribute attribute{};
        attribute.id = cudaLaunchAttributeClusterDimension;
        attribute.val.clusterDim.x = 2;
        attribute.val.clusterDim.y = 1;
        attribute.val.clusterDim.z = 1;
        config.attrs = &attribute;
        config.numAttrs = 1;
        int clusters = 0;
        st = cudaOccupancyMaxActiveClusters(&clusters, tc2_kernels[i].first, &config);
        if (st != cudaSuccess) {
            cudaGetLastError();
            clusters = 0;
        }
        if (ctx->max_pairs < 0 || clusters < ctx->max_pairs)
            ctx->max_pairs = clusters;
    }
    // ... and how many CTAs of the single-CTA kernel in split-K clusters of 2, 4, 8.
    ctx->max_split_ctas[0] = ctx->sm_count;
    for (int i = 1; i < 4; ++i) {
        const unsigned int size = 1u << i;
        cudaLaunchConfig_t config{};
        config.gridDim = dim3(1, 1, size);
        config.blockDim = dim3(TC_THREADS, 1, 1);
        config.dynamicSmemBytes = TcTile<256>::kSmem;
        cudaLaunchAttribute attribute{};
        attribute.id = cudaLaunchAttributeClusterDimension;
        attribute.val.clusterDim.x = 1;
        attribute.val.clusterDim.y = 1;
        attribute.val.clusterDim.z = size;
        config.attrs = &attribute;
        config.numAttrs = 1;
        int clusters = 0;
        st = cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void *>(&tc_gemm_kernel<kFmtBF16, 256>),
                                            &config);
        if (st != cudaSuccess) {
            cudaGetLastError();
            clusters = 0;
        }
        ctx->max_split_ctas[i] = clusters * static_cast<int>(size);
    }
    ctx->device_sm_count = ctx->sm_count;
    ctx->device_max_pairs = ctx->max_pairs;
    for (int i = 0; i < 4; ++i)
        ctx->device_max_split_ctas[i] = ctx->max_split_ctas[i];

    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    st = cudaMemPoolCreate(&ctx->pool, &props);
    if (st == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep);
    } else {
        ctx->pool = nullptr;
        cudaGetLastError();
    }
    return ctx;
}

extern "C" int matmul_destroy(void *opaque, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_destroy", "context is null");
    Context *ctx = static_cast<Context *>(opaque);
    const cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    if (ctx->pool) {
        // Outstanding stream-ordered frees must retire before the pool goes away.
        cudaDeviceSynchronize();
        cudaMemPoolDestroy(ctx->pool);
        cudaGetLastError();
    }
    delete ctx;
    return 0;
}

extern "C" int matmul_launch(void *opaque, int implementation, int precision, const void *a, const void *b,
                             float *c, int m, int k, int n, void *stream, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_launch", "context is null");
    if (!a || !b || !c)
        return fail(error, error_size, "matmul_launch", "matrix pointer is null");
    if (m <= 0 || k <= 0 || n <= 0)
        return fail(error, error_size, "matmul_launch", "dimensions must be positive");
    if (check_ids(implementation, precision, "matmul_launch", error, error_size))
        return 1;
    const size_t elem = precision == kPrecFp16 || precision == kPrecBf16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % elem ||
        reinterpret_cast<uintptr_t>(c) % 4)
        return fail(error, error_size, "matmul_launch", "matrix pointer is not aligned to its element size");
    Context *ctx = static_cast<Context *>(opaque);
    const cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (implementation == kImplFfma)
        return launch_ffma(ctx, static_cast<const float *>(a), static_cast<const float *>(b), c, m, k, n, s, error,
                           error_size);
    return launch_tcgen05(ctx, precision, a, b, c, m, k, n, s, error, error_size);
}

extern "C" int matmul_plan(void *opaque, int implementation, int precision, int m, int k, int n, char *json,
                           size_t json_size, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (json && json_size)
        json[0] = '\0';
    if (!opaque)
        return fail(error, error_size, "matmul_plan", "context is null");
    if (!json || json_size == 0)
        return fail(error, error_size, "matmul_plan", "JSON buffer is null");
    if (m <= 0 || k <= 0 || n <= 0)
        return fail(error, error_size, "matmul_plan", "dimensions must be positive");
    if (check_ids(implementation, precision, "matmul_plan", error, error_size))
        return 1;
    const Context *ctx = static_cast<const Context *>(opaque);
    int written;
    if (implementation == kImplFfma) {
        // One kernel for every alignment; the plan does not depend on the base pointers.
        const FfmaPlan plan = choose_ffma_plan(m, k, n, ctx->sm_count, ctx->ffma_resident);
        const FfmaTileOption &o = kFfmaTiles[plan.tile];
        written = std::snprintf(json, json_size,
                                "{\"kernel\":\"ffma_async\",\"tile_m\":%d,\"tile_n\":%d,\"threads\":%d,"
                                "\"splits\":%d,\"cluster\":[1,1,%d],\"grid\":[%lld,%lld,%d],"
                                "\"vector_loads_if_aligned\":%s,\"staging_if_aligned\":\"%s\"}",
                                o.bm, o.bn, o.warps * 32, plan.splits, plan.splits,
                                static_cast<long long>((n + o.bn - 1) / o.bn),
                                static_cast<long long>((m + o.bm - 1) / o.bm), plan.splits,
                                k % 4 == 0 && n % 4 == 0 ? "true" : "false",
                                k % 4 == 0 && n % 4 == 0 ? (plan.tile == 0 ? "tma" : "cp_async16") : "cp_async4");
    } else if (precision == kPrecTf32 && tf32_on_ffma(m, k, n)) {
        const FfmaPlan plan = choose_ffma_plan(m, k, n, ctx->sm_count, ctx->ffma_resident, 2u);
        written = std::snprintf(json, json_size,
                                "{\"kernel\":\"ffma_tf32_rne\",\"tile_m\":32,\"tile_n\":32,\"threads\":64,"
                                "\"splits\":%d,\"cluster\":[1,1,%d]}",
                                plan.splits, plan.splits);
    } else if (m <= kSkinnyMaxM) {
        const int elem = precision == kPrecTf32 ? 4 : 2;
        const int total_k_blocks = static_cast<int>((static_cast<int64_t>(k) + TC_ROW_BYTES / elem - 1) /
                                                    (TC_ROW_BYTES / elem));
        written = std::snprintf(json, json_size,
                                "{\"kernel\":\"tc_skinny\",\"tile_m\":%d,\"tile_n\":%d,\"splits\":%d}",
                                m <= 16 ? 16 : m <= 32 ? 32 : 64, SK_BM, skinny_splits(ctx, n, total_k_blocks));
    } else {
        const TcPlan plan = choose_tc_plan(ctx, m, k, n, precision);
        const bool pair = plan.tile_n == 0 || plan.tile_n == TC2W_BN;
        const int tile_m = pair ? TC2_BM : TC_BM;
        const int tile_n = plan.tile_n == 0 ? TC2_BN : plan.tile_n;
        const int64_t tiles = ((static_cast<int64_t>(m) + tile_m - 1) / tile_m) *
                              ((static_cast<int64_t>(n) + tile_n - 1) / tile_n);
        const int64_t ctas = pair ? 2 * (tiles < ctx->max_pairs ? tiles : ctx->max_pairs)
                             : plan.splits > 1 ? tiles * plan.splits
                                               : (tiles < ctx->sm_count ? tiles : ctx->sm_count);
        written = pair
                      ? std::snprintf(json, json_size,
                                      "{\"kernel\":\"tc2_pair\",\"tile_m\":%d,\"tile_n\":%d,\"cluster\":[2,1,1],"
                                      "\"splits\":1,\"ctas\":%lld}",
                                      TC2_BM, tile_n, static_cast<long long>(ctas))
                      : std::snprintf(json, json_size,
                                      "{\"kernel\":\"tc_single\",\"tile_m\":%d,\"tile_n\":%d,\"splits\":%d,"
                                      "\"cluster\":[1,1,%d],\"ctas\":%lld}",
                                      TC_BM, plan.tile_n, plan.splits, plan.splits, static_cast<long long>(ctas));
    }
    if (written < 0 || static_cast<size_t>(written) >= json_size) {
        json[0] = '\0';
        return fail(error, error_size, "matmul_plan", "JSON buffer too small");
    }
    return 0;
}

extern "C" int matmul_set_sm_limit(void *opaque, int sms, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_set_sm_limit", "context is null");
    Context *ctx = static_cast<Context *>(opaque);
    if (sms < 0 || (sms > 0 && sms < 2))
        return fail(error, error_size, "matmul_set_sm_limit", "the limit must be 0 (no limit) or at least 2 SMs");
    const int limit = sms == 0 || sms > ctx->device_sm_count ? ctx->device_sm_count : sms;
    ctx->sm_count = limit;
    ctx->max_pairs = ctx->device_max_pairs < limit / 2 ? ctx->device_max_pairs : limit / 2;
    for (int i = 0; i < 4; ++i) {
        const int whole = limit / (1 << i) * (1 << i);
        ctx->max_split_ctas[i] = ctx->device_max_split_ctas[i] < whole ? ctx->device_max_split_ctas[i] : whole;
    }
    return 0;
}

extern "C" int matmul_set_wait_limit(void *opaque, unsigned long long nanoseconds, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_set_wait_limit", "context is null");
    if (nanoseconds > kWaitLimitNs)
        return fail(error, error_size, "matmul_set_wait_limit", "the limit cannot exceed 2 s (2000000000 ns)");
    static_cast<Context *>(opaque)->wait_limit_ns = nanoseconds;
    return 0;
}

extern "C" int matmul_peer_push(void *opaque, const void *src, void *const *peer_dst, int peers, size_t bytes,
                                int ctas, void *stream, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_peer_push", "context is null");
    if (peers < 0 || peers > PP_MAX_PEERS)
        return fail(error, error_size, "matmul_peer_push", "peers must be between 0 and 7");
    if (bytes % 16 != 0)
        return fail(error, error_size, "matmul_peer_push", "the block size must be a multiple of 16 bytes");
    if (ctas < 0)
        return fail(error, error_size, "matmul_peer_push", "ctas must be 0 (the default) or positive");
    if (peers == 0 || bytes == 0)
        return 0;
    if (!src || !peer_dst || !aligned16(src))
        return fail(error, error_size, "matmul_peer_push", "source is null or not 16-byte aligned");
    PeerPushJob job{};
    job.src = static_cast<const float4 *>(src);
    job.peers = peers;
    job.count = static_cast<long long>(bytes / 16);
    for (int p = 0; p < peers; ++p) {
        if (!peer_dst[p] || !aligned16(peer_dst[p]))
            return fail(error, error_size, "matmul_peer_push", "a destination is null or not 16-byte aligned");
        job.dst[p] = static_cast<float4 *>(peer_dst[p]);
    }
    Context *ctx = static_cast<Context *>(opaque);
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    const long long needed = (job.count + PP_THREADS - 1) / PP_THREADS;
    const int grid = static_cast<int>(needed < (ctas ? ctas : 16) ? needed : (ctas ? ctas : 16));
    peer_push_kernel<<<grid, PP_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(job);
    st = cudaGetLastError();
    if (st != cudaSuccess)
        return fail(error, error_size, "matmul_peer_push", cudaGetErrorString(st));
    return 0;
}

extern "C" int matmul_convert(void *opaque, int precision, const float *src, void *dst, size_t count, void *stream,
                              char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_convert", "context is null");
    if (precision < 0 || precision > 3)
        return fail(error, error_size, "matmul_convert", "unknown precision");
    if (!src || !dst)
        return fail(error, error_size, "matmul_convert", "pointer is null");
    if (count == 0)
        return 0;
    Context *ctx = static_cast<Context *>(opaque);
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t n = static_cast<int64_t>(count);
    const int64_t blocks = (n + 255) / 256;
    const unsigned int grid = static_cast<unsigned int>(blocks < 16LL * ctx->sm_count ? blocks : 16LL * ctx->sm_count);
    if (precision == kPrecFp32)
        st = cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyDeviceToDevice, s);
    else if (precision == kPrecTf32)
        convert_f32_kernel<float><<<grid, 256, 0, s>>>(src, static_cast<float *>(dst), n);
    else if (precision == kPrecBf16)
        convert_f32_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(src, static_cast<__nv_bfloat16 *>(dst), n);
    else
        convert_f32_kernel<__half><<<grid, 256, 0, s>>>(src, static_cast<__half *>(dst), n);
    if (st == cudaSuccess)
        st = cudaGetLastError();
    if (st != cudaSuccess)
        return fail(error, error_size, "matmul_convert", cudaGetErrorString(st));
    return 0;
}

extern "C" int matmul_device_status(void *opaque, int clear, unsigned int *status, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_device_status", "context is null");
    if (!status)
        return fail(error, error_size, "matmul_device_status", "status pointer is null");
    Context *ctx = static_cast<Context *>(opaque);
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st == cudaSuccess)
        st = cudaDeviceSynchronize();
    if (st == cudaSuccess)
        st = cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned int));
    if (st == cudaSuccess && clear) {
        const unsigned int zero = 0;
        st = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int));
    }
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "matmul_device_status", st);
    return 0;
}

extern "C" int matmul_launch_noalloc(void *opaque, int implementation, int precision, const void *a,
                                     const void *b, float *c, int m, int k, int n, void *stream, char *error,
                                     size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_launch_noalloc", "context is null");
    if (!a || !b || !c)
        return fail(error, error_size, "matmul_launch_noalloc", "matrix pointer is null");
    if (m <= 0 || k <= 0 || n <= 0)
        return fail(error, error_size, "matmul_launch_noalloc", "dimensions must be positive");
    if (check_ids(implementation, precision, "matmul_launch_noalloc", error, error_size))
        return 1;
    if (implementation != kImplTcgen05)
        return fail(error, error_size, "matmul_launch_noalloc",
                    "only implementation 7 (tcgen05) has a fixed-scratch variant; the FFMA kernel needs no "
                    "scratch, use matmul_launch");
    const size_t elem = precision == kPrecFp16 || precision == kPrecBf16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % elem ||
        reinterpret_cast<uintptr_t>(c) % 4)
        return fail(error, error_size, "matmul_launch_noalloc", "matrix pointer is not aligned to its element size");
    Context *ctx = static_cast<Context *>(opaque);
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    void *scratch = nullptr;
    st = noalloc_scratch_address(ctx, &scratch);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "matmul_launch_noalloc: cudaGetSymbolAddress", st);
    return launch_tcgen05(ctx, precision, a, b, c, m, k, n, static_cast<cudaStream_t>(stream), error, error_size,
                          scratch, kNoAllocScratchBytes);
}

extern "C" int matmul_check_fp64(void *opaque, int precision, const void *a, const void *b, const float *c, int m,
                                 int k, int n, void *stream, double *result, char *error, size_t error_size)
{
    clear_error(error, error_size);
    if (!opaque)
        return fail(error, error_size, "matmul_check_fp64", "context is null");
    if (!a || !b || !c || !result)
        return fail(error, error_size, "matmul_check_fp64", "pointer is null");
    if (m <= 0 || k <= 0 || n <= 0)
        return fail(error, error_size, "matmul_check_fp64", "dimensions must be positive");
    if (precision < 0 || precision > 3)
        return fail(error, error_size, "matmul_check_fp64", "unknown precision");
    Context *ctx = static_cast<Context *>(opaque);
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "cudaSetDevice", st);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // gamma_K for u = 2^-23, as in the reference's GemmReference.
    const double u = std::ldexp(1.0, -23);
    const double ku = static_cast<double>(k) * u;
    const double gamma = ku < 1.0 ? ku / (1.0 - ku) : std::expm1(static_cast<double>(k) * std::log1p(u));
    const unsigned long long zero[2] = {0ull, 0ull};
    st = cudaMemcpyToSymbolAsync(g_check_result, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "matmul_check_fp64", st);
    const int64_t tiles = ((m + CK_TILE - 1) / CK_TILE) * static_cast<int64_t>((n + CK_TILE - 1) / CK_TILE);
    const int grid = static_cast<int>(tiles < 8LL * ctx->sm_count ? tiles : 8LL * ctx->sm_count);
    if (precision == kPrecFp32)
        fp64_check_kernel<float, false><<<grid, 256, 0, s>>>(static_cast<const float *>(a),
                                                             static_cast<const float *>(b), c, m, n, k, gamma);
    else if (precision == kPrecTf32)
        fp64_check_kernel<float, true><<<grid, 256, 0, s>>>(static_cast<const float *>(a),
                                                            static_cast<const float *>(b), c, m, n, k, gamma);
    else if (precision == kPrecBf16)
        fp64_check_kernel<__nv_bfloat16, false><<<grid, 256, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(a), static_cast<const __nv_bfloat16 *>(b), c, m, n, k, gamma);
    else
        fp64_check_kernel<__half, false><<<grid, 256, 0, s>>>(static_cast<const __half *>(a),
                                                              static_cast<const __half *>(b), c, m, n, k, gamma);
    st = cudaGetLastError();
    unsigned long long bits[2] = {0ull, 0ull};
    if (st == cudaSuccess)
        st = cudaMemcpyFromSymbolAsync(bits, g_check_result, sizeof(bits), 0, cudaMemcpyDeviceToHost, s);
    if (st == cudaSuccess)
        st = cudaStreamSynchronize(s);
    if (st != cudaSuccess)
        return fail_cuda(error, error_size, "matmul_check_fp64", st);
    std::memcpy(&result[0], &bits[0], sizeof(double));
    std::memcpy(&result[1], &bits[1], sizeof(double));
    return 0;
}
