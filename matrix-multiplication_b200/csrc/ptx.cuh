// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA (cp.async.bulk.tensor),
// tcgen05 (TMEM allocation, MMA, commit, loads) and proxy fences.
//
// Every wait on an mbarrier goes through mbar_wait(), which polls with
// try_wait and gives up after a limit of %globaltimer time so that a protocol
// error ends the kernel with a status flag instead of hanging the GPU.  Two
// kinds of wait:
//   * progress waits (a stage to land, an accumulator to fill or drain) use
//     the launch's limit, kWaitLimitNs unless matmul_set_wait_limit lowered it;
//   * drain waits (copies and MMAs this CTA or its pair has already issued,
//     which always complete) keep kWaitLimitNs, so that no CTA can leave while
//     a copy into its shared memory or an MMA on its TMEM is still in flight.
#pragma once

#include <cstdint>

namespace b200 {

// Longest legitimate wait in these kernels is one output tile's full K loop
// (milliseconds even for K in the millions); two seconds means a broken protocol.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels launched with programmatic stream serialisation start while the
// previous kernel on the stream is still finishing; each of ours runs its
// prologue (barriers, TMEM, descriptor prefetch), then waits here for the
// previous kernel to complete with its memory visible before touching global
// memory.  A kernel launched without the attribute returns at once.
__device__ __forceinline__ void wait_for_prior_grid()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next kernel on the stream begin its own prologue on SMs this grid
// frees; it still waits for this grid's completion before reading memory.
__device__ __forceinline__ void allow_next_grid()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking test of the phase with the given parity (no suspension).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Limits below this are watchdog settings (matmul_set_wait_limit): they poll
// with test_wait, which never suspends, so that even a wait shorter than
// try_wait's own suspension (one TMA stage) can run out.
constexpr uint64_t kShortWaitNs = 1000000ull;

// Waits until the phase with the given parity has completed.  Returns false
// (without waiting further) once `limit_ns` has passed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs)
{
    if (limit_ns < kShortWaitNs) {
        const uint64_t start = global_timer_ns();
        for (;;) {
            if (mbar_test_wait(bar, parity))
                return true;
            // %globaltimer advances in steps of up to a microsecond: a limit below that
            // allows one test.
            if (limit_ns < 1000u || global_timer_ns() - start > limit_ns)
                return false;
        }
    }
    if (mbar_try_wait(bar, parity))
        return true;
    // try_wait itself suspends the thread for a while before it reports "not yet",
    // so reading the timer after every poll costs nothing that matters and keeps
    // a short limit honoured.
    const uint64_t start = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity))
            return true;
        if (global_timer_ns() - start > limit_ns)
            return false;
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_map(const void *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completion is signalled to
// `bar` as transaction bytes (the full box size, out-of-bounds parts zero-filled).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *map, uint32_t bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// 2-D tiled store of one box from shared memory (out-of-bounds parts clipped).
__device__ __forceinline__ void tma_store_2d(const void *map, uint32_t src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group()
{
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N committed bulk groups are incomplete (writes visible).
template <int N>
__device__ __forceinline__ void bulk_wait_group()
{
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy.
__device__ __forceinline__ void fence_proxy_async_shared()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// ---------------------------------------------------------------- epilogue warpgroup
// The four epilogue warps (128 threads) synchronise on named barrier 1; warps
// of other roles never touch it.
__device__ __forceinline__ void epilogue_sync()
{
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// 1 only if every epilogue thread passes 1: the four warps then take the same
// branch, so none of them can be left waiting at barrier 1 for a warp that left.
__device__ __forceinline__ int epilogue_all(int ok)
{
    uint32_t all;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(all)
        : "r"(static_cast<uint32_t>(ok))
        : "memory");
    return static_cast<int>(all);
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t columns)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                 "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], one instruction, issued by one thread.
template <bool TF32>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate)
{
    if constexpr (TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Load 32 consecutive FP32 columns of this thread's TMEM lane (32x32b shape,
// 32 repetitions) and wait for completion in the same asm block so that no
// consumer of the registers can be scheduled before the wait.
__device__ __forceinline__ void tmem_load_32cols(uint32_t taddr, uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
__device__ __forceinline__ uint32_t cluster_cta_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t addr, uint32_t rank)
{
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
    return out;
}

// Arrive on an mbarrier that may live in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 16-byte load from the shared memory of a CTA of this cluster (a mapa address).
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t cluster_addr)
{
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cluster_addr)
                 : "memory");
    return v;
}

// 4-byte load from the shared memory of a CTA of this cluster (a mapa address).
__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t cluster_addr)
{
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
    return v;
}

// 16-byte store into the shared memory of a CTA of this cluster (a mapa address).
__device__ __forceinline__ void st_shared_cluster_v4(uint32_t cluster_addr, uint32_t a, uint32_t b, uint32_t c,
                                                     uint32_t d)
{
    asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory into a
// CTA of this cluster (`dst` and its mbarrier `bar` are mapa addresses); the
// destination mbarrier receives the byte count as complete_tx.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst),
                 "r"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Every thread of every CTA in the cluster.
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is signalled
// to an mbarrier of either CTA of the pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *map, uint32_t bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot, uint32_t columns)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t columns)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

// D[tmem of both CTAs] (+)= A[both CTAs' smem] * B[both CTAs' smem], issued by the pair's leader.
template <bool TF32>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate)
{
    if constexpr (TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrive once on the mbarrier at shared::cluster address `bar` (this CTA's or
// the peer's) when every pair MMA issued so far by this thread is done.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// The same completion signal delivered to the mbarrier at offset `bar` in every
// CTA of `cta_mask` with one instruction (a commit, not a data load: nothing is
// read from any CTA's memory).  One arrival per pair stage instead of two
// separate commits keeps the MMA issue stream dense.
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar, uint16_t cta_mask)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     bar),
                 "h"(cta_mask)
                 : "memory");
}

// L2 policy for data that will not be read again soon (the FP32 output).
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// 2-D tiled store with an L2 cache-policy hint.
__device__ __forceinline__ void tma_store_2d_hint(const void *map, uint32_t src, int x, int y, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// 16 consecutive FP32 columns of this thread's TMEM lane, waited in the same asm block.
__device__ __forceinline__ void tmem_load_16cols(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma (sm_100 format, version 1):
// start address, leading- and stride-dimension byte offsets (all >> 4) and the
// swizzle layout in bits 61-63: 2 = 128-byte swizzle (16-byte chunks XOR row % 8
// over 8 rows of 128 bytes), 1 = 128-byte swizzle with 32-byte atoms (32-byte
// chunks XOR row % 4 over 4 rows of 128 bytes), the form an MN-major TF32
// operand takes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout_type)
{
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    desc |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    desc |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    desc |= 1ull << 46;
    desc |= static_cast<uint64_t>(layout_type & 7u) << 61;
    return desc;
}

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes)
{
    return smem_desc(addr, lbo_bytes, sbo_bytes, 2u);
}

// Descriptor of an MN-major operand staged as boxes of 128-byte rows (one row
// per k, kBK rows per box), consecutive boxes `box_bytes` apart along M/N.
// FP16/BF16: 128-byte swizzle, 8-row atoms (stride-dimension offset 1024);
// TF32: 32-byte-atom swizzle, 4-row atoms (offset 512).  The leading-dimension
// offset is the distance between boxes.
template <bool TF32>
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr, uint32_t box_bytes)
{
    return TF32 ? smem_desc(addr, box_bytes, 512u, 1u) : smem_desc(addr, box_bytes, 1024u, 2u);
}

} // namespace b200
