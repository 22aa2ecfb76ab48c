// ptx.cuh — the sm_100a primitives every e2cuda kernel is built from: mbarriers with bounded
// waits, TMA tile loads (never multicast), and the tcgen05 tensor-memory / MMA instructions.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define E2C_DEV __device__ __forceinline__

// A wait that has not completed after this long is a failure: the kernel records it in the status
// word and unwinds instead of hanging the GPU.
#ifndef E2C_WAIT_NS
#define E2C_WAIT_NS 2000000000ull
#endif

// Status codes a kernel can leave in the status word (first failure wins).
enum {
    E2C_OK = 0,
    E2C_ERR_WAIT_PRODUCER = 0x101,  // TMA producer gave up waiting for a free stage
    E2C_ERR_WAIT_MMA = 0x102,       // MMA issuer gave up waiting for operands / accumulator
    E2C_ERR_WAIT_EPI = 0x103,       // epilogue gave up waiting for an accumulator
    E2C_ERR_WAIT_ATTN = 0x104,      // attention softmax / correction gave up
    E2C_ERR_WAIT_DRAIN = 0x105,     // teardown gave up draining in-flight copies
    E2C_ERR_BAD_TOKEN = 0x106,      // a token id outside the table (row 0 used instead)
    E2C_ERR_SMEM_ALIGN = 0x107      // dynamic shared memory not 1024-byte aligned: the kernel did nothing
};

E2C_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

E2C_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch. A kernel launched with the programmatic-serialization attribute
// may start while the previous kernel of its stream is still running: it must pass griddep_wait(),
// which returns once that kernel (and so every earlier one) has finished and its writes are
// visible, before it reads or writes global memory the stream's earlier kernels touch. For a kernel
// launched without the attribute both calls do nothing. griddep_launch_dependents() lets the next
// kernel of the stream be scheduled as soon as SMs free up.
E2C_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
E2C_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

E2C_DEV void record_status(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------------------- mbarrier
E2C_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
E2C_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
E2C_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
                 : "memory");
}
E2C_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
E2C_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// The same, but the thread may sleep in the instruction until the phase completes or `ns`
// nanoseconds have passed: a waiting warp issues nothing meanwhile, so the warps that are working
// keep the issue slots.
E2C_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
// Longest sleep of one wait step; the failure checks below run between steps.
#ifndef E2C_WAIT_STEP_NS
#define E2C_WAIT_STEP_NS 100000u
#endif
// A wait reads the kernel's status word (another role's failure) only once it has lasted this
// long: the read is a global load, and a barrier that completes while it is in flight would wake
// the waiter a memory round trip late. Waits of a working pipeline end well before this.
#ifndef E2C_WAIT_POLL_NS
#define E2C_WAIT_POLL_NS 20000ull
#endif
// Wait until the phase with parity `parity` has completed. Bounded: returns false (and records
// `code`) after E2C_WAIT_NS, or soon after another role of this kernel has failed.
E2C_DEV bool mbar_wait(uint32_t bar, uint32_t parity, int *status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, E2C_WAIT_STEP_NS)) return true;
        const uint64_t dt = globaltimer() - t0;
        if (dt > E2C_WAIT_NS) {
            record_status(status, code);
            return false;
        }
        if (dt > E2C_WAIT_POLL_NS && status && *(volatile int *)status != 0) return false;
    }
}

// ------------------------------------------------------------------------------- TMA
E2C_DEV void tma_prefetch_desc(const CUtensorMap *m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2D tile load into this CTA's shared memory, completion counted on `bar` in bytes. The x
// coordinate (innermost, bytes = x * elem) must be 16-byte aligned.
E2C_DEV void tma_load_2d(uint32_t dst, const CUtensorMap *m, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// 2D tile store from this CTA's shared memory (bulk-group completion). Rows / columns outside the
// tensor are not written.
E2C_DEV void tma_store_2d(const CUtensorMap *m, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}
E2C_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of every committed store have been read (the buffer may be rewritten)
E2C_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the same for all but the most recently committed group
E2C_DEV void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
E2C_DEV void bulk_wait_read2() { asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); }
// every committed store has completed
E2C_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// 4 bytes global -> shared without a register round trip; src_bytes 0 writes a zero and reads
// nothing. Visible to the issuing thread after cp_async_wait_all().
E2C_DEV void cp_async_4(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
E2C_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
E2C_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// every group but the most recently committed one has landed
E2C_DEV void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
E2C_DEV void named_barrier(int id, int nthreads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory"); }
// named barrier that also returns whether `pred` held in every participating thread
E2C_DEV bool named_barrier_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// generic-proxy shared-memory writes become visible to the async proxy (tcgen05.mma operands)
E2C_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------- tcgen05
E2C_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
E2C_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
E2C_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// The same for a CTA pair (cta_group::2): issued by the same warp in both CTAs of the cluster, which
// then hold the same TMEM address.
E2C_DEV void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
E2C_DEV void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
E2C_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
E2C_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
E2C_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32 (kind::i8), one thread issues.
E2C_DEV void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// bf16 x bf16 -> fp32 (kind::f16), one thread issues.
E2C_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// bf16 x bf16 -> fp32 with the A operand (M = 128 rows x K = 16, two bf16 per 32-bit column) read
// from tensor memory at a_tmem; B from shared memory as above.
E2C_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
        : "memory");
}
// Arrive once on `bar` when every tcgen05.mma this thread issued so far has completed.
E2C_DEV void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// ------------------------------------------------------------------------------- CTA pairs
// A pair of CTAs (a cluster of two) runs one M = 256 product: each CTA holds 128 rows of A and half
// of B's N rows in its shared memory, and 128 rows x N of the accumulator in its TMEM. The MMA and
// its commits are issued by the CTA of rank 0 (the leader) only.
E2C_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the shared::cluster address of the variable at shared::cta address `addr` in the CTA of `rank`
E2C_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// every thread of both CTAs (release / acquire at cluster scope); the non-.aligned forms, so that
// warps whose lanes arrive at different times (one elected lane did the role's work) are fine
E2C_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// arrive on an mbarrier given by its shared::cluster address (possibly in the other CTA), with
// the default semantics (release at CTA scope); cluster-scope release made every arrival wait for
// the thread's earlier writes and stalled the epilogue between tiles
E2C_DEV void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// the same with release semantics at cluster scope: the arriving thread's earlier writes (to this
// CTA's or another's shared memory) are visible to a thread that then waits with acquire.cluster
E2C_DEV void mbar_arrive_cluster_release(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
E2C_DEV bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait with acquire at cluster scope (pairs with mbar_arrive_cluster_release)
E2C_DEV bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int *status, int code) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(E2C_WAIT_STEP_NS)
            : "memory");
        if (ok) return true;
        const uint64_t dt = globaltimer() - t0;
        if (dt > E2C_WAIT_NS) {
            record_status(status, code);
            return false;
        }
        if (dt > E2C_WAIT_POLL_NS && status && *(volatile int *)status != 0) return false;
    }
}
// Asynchronous stores into another CTA's shared memory whose bytes complete on an mbarrier of that
// CTA (like a TMA load's): the receiver expects the bytes with mbar_arrive_expect_tx and waits on
// the barrier; no release fence on the sender's side.
E2C_DEV void st_async_f32(uint32_t cluster_addr, float v, uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(cluster_addr), "f"(v),
                 "r"(cluster_bar)
                 : "memory");
}
E2C_DEV void st_async_f32x2(uint32_t cluster_addr, float a, float b, uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(cluster_addr),
                 "f"(a), "f"(b), "r"(cluster_bar)
                 : "memory");
}
E2C_DEV void st_dsmem_f32(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
E2C_DEV void st_dsmem_f32x2(uint32_t cluster_addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(cluster_addr), "f"(a), "f"(b) : "memory");
}
// 2D tiled TMA load into this CTA's shared memory whose completed bytes are counted on the
// mbarrier `bar_cluster` (a shared::cluster address: the leader's barrier). No multicast.
E2C_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap *m, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
// M = 256 int8 product over the pair: A and B descriptors address the leader's shared memory; the
// same offsets in the other CTA hold its rows of A and its half of B.
E2C_DEV void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at shared::cluster address `bar_cluster` when every pair MMA this
// thread issued so far has completed.
E2C_DEV void mma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

// K-major operand tile in shared memory with the 128-byte swizzle: rows of 128 bytes, 8-row
// groups 1024 bytes apart (SBO), the leading offset unused. Base must be 1024-byte aligned; a
// k-step inside the 128-byte row advances the start address.
E2C_DEV uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset
    d |= (uint64_t)1 << 46;              // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;              // SWIZZLE_128B
    return d;
}

// The same for K-major tiles whose rows are 64 bytes, stored with the 64-byte swizzle (8-row groups
// 512 bytes apart; layout type 4 = SWIZZLE_64B).
E2C_DEV uint64_t smem_desc_sw64(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(512u >> 4) << 32;  // stride byte offset
    d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
    d |= (uint64_t)4 << 61;             // SWIZZLE_64B
    return d;
}

// Instruction descriptors (M = 128, K-major A and B, dense).
__host__ __device__ constexpr uint32_t idesc_i8(int n, int m = 128) {
    return (2u << 4)            // D = s32
           | (1u << 7)          // A = s8
           | (1u << 10)         // B = s8
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4)            // D = f32
           | (1u << 7)          // A = bf16
           | (1u << 10)         // B = bf16
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets row (lane quadrant*32 + t).
E2C_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
E2C_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns
E2C_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns
E2C_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
E2C_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
E2C_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
E2C_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

E2C_DEV uint32_t elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred;
}
