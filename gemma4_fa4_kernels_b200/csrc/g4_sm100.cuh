// Blackwell (sm_100a) building blocks shared by the attention kernels:
// mbarriers with bounded waits, TMA tile loads, and tcgen05 tensor-core /
// tensor-memory (TMEM) primitives written as inline PTX.
//
// Conventions used by every kernel in this library:
//  * operand tiles live in shared memory in the 128-byte-swizzled layout that
//    a TMA load with CU_TENSOR_MAP_SWIZZLE_128B produces: 64 bf16 (128 B) per
//    row, 8-row atoms of 1024 B, every tile base 1024-B aligned;
//  * one such tile can be described to the tensor core either K-major (rows =
//    M/N index, 64 contiguous K values per row) or MN-major (rows = K index,
//    64 contiguous M/N values per row) -- the same bytes serve both roles;
//  * accumulators are fp32 in TMEM, M = 128: row i is TMEM lane i;
//  * a bf16 A operand held in TMEM packs two consecutive K values per
//    32-bit column (K = 16 per MMA -> 8 columns).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace g4 {

// ------------------------------------------------------------------------------------
// error reporting (device side): the first failure wins, later ones are dropped
// ------------------------------------------------------------------------------------
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutTma = 1,     // a TMA transaction never completed
  kDevTimeoutMma = 2,     // an MMA commit never arrived
  kDevTimeoutPeer = 3,    // a producer/consumer role never signalled
};

// Wall-clock bound on any single wait (ns).  Far above any legitimate wait.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Shared per-CTA abort word: once any role times out, every other wait returns
// false promptly so that the CTA can reach its teardown (TMEM release).
struct CtaAbort {
  volatile int* flag;   // shared memory
  int* error;           // global error word (may be null)
};

// Wait until the phase with the given parity has completed.  Returns false
// (after recording `code`) if the wait exceeds kWaitLimitNs or the CTA aborts.
// The poll loop sits inside one PTX block, bounded by %globaltimer and by the
// CTA abort word; the timer is read only after a failed first try.  Measured
// with a tcgen05.mma issue probe (M128 N128 K16, a wait per 8 MMAs): an issuing
// thread that polls through a C++ loop around try_wait issues an MMA every 135
// cycles, a converged warp polling here every 70 (the tensor pipe needs 68).
// Any caller may use it (one lane or a whole warp); lanes of a converged warp
// all return the same value.
#define G4_WAIT_ASM(TRY)                                                              \
  asm volatile(                                                                       \
      "{\n\t.reg .pred p;\n\t.reg .u64 t0, t1;\n\t.reg .u32 f;\n\t"                   \
      TRY " p, [%1], %2;\n\t"                                                         \
      "@p bra LAB_DONE;\n\t"                                                          \
      "mov.u64 t0, %%globaltimer;\n"                                                  \
      "LAB_WAIT:\n\t"                                                                 \
      TRY " p, [%1], %2;\n\t"                                                         \
      "@p bra LAB_DONE;\n\t"                                                          \
      "ld.volatile.shared.u32 f, [%3];\n\t"                                           \
      "setp.ne.u32 p, f, 0;\n\t"                                                      \
      "@p bra LAB_FAIL;\n\t"                                                          \
      "mov.u64 t1, %%globaltimer;\n\t"                                                \
      "sub.u64 t1, t1, t0;\n\t"                                                       \
      "setp.lt.u64 p, t1, %4;\n\t"                                                    \
      "@p bra LAB_WAIT;\n"                                                            \
      "LAB_FAIL:\n\t"                                                                 \
      "setp.ne.u32 p, 0, 0;\n"                                                        \
      "LAB_DONE:\n\t"                                                                 \
      "selp.u32 %0, 1, 0, p;\n\t}"                                                    \
      : "=r"(done)                                                                    \
      : "r"(smem_addr(bar)), "r"(parity), "r"(smem_addr((const void*)ab.flag)),       \
        "l"(kWaitLimitNs)                                                             \
      : "memory")

// One lane of a converged warp (elect.sync over the full mask): the lowest
// active lane, so every call in a converged warp elects lane 0.
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(e));
  return e != 0;
}

// AND of `pred` over the `count` threads that meet on named barrier `id`
// (bar.red.and): every participant gets the same answer, so a branch on it is
// uniform across them even when `pred` differs between their warps.
__device__ __forceinline__ bool bar_red_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ bool wait_fail(const CtaAbort& ab, int code) {
  if (!*ab.flag) {  // this wait ran out of time (not an abort raised elsewhere)
    *ab.flag = 1;
    if (ab.error) atomicCAS(ab.error, 0, code);
  }
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const CtaAbort& ab,
                                          int code) {
  uint32_t done;
  G4_WAIT_ASM("mbarrier.try_wait.parity.shared::cta.b64");
  return done ? true : wait_fail(ab, code);
}
// The same with cluster-scope acquire (barriers that receive peer-CTA arrivals).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  const CtaAbort& ab, int code) {
  uint32_t done;
  G4_WAIT_ASM("mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64");
  return done ? true : wait_fail(ab, code);
}

// ------------------------------------------------------------------------------------
// CTA pairs: 2-CTA clusters whose tensor-core work is issued as tcgen05
// cta_group::2 operations by the even (leader) CTA
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs: prior shared-memory writes (barrier inits
// included) become visible cluster-wide.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
// shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (any CTA of the
// cluster), releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr)
               : "memory");
}
// ------------------------------------------------------------------------------------
// TMA: every load delivers into the issuing CTA's own shared memory
// ------------------------------------------------------------------------------------
// Pair forms of the tiled loads: the box lands in this CTA's shared memory and
// its bytes complete on the leader CTA's mbarrier (`leader_bar`, a
// shared::cluster address), so one barrier tracks both halves of a pair-wide
// operand stage.
__device__ __forceinline__ void tma_load_4d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int c0, int c1, int c2,
                                                 int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled load: coordinates (c0 = head-dim element, c1 = head, c2 = token, c3 = batch).
// c0 is always a multiple of 64 elements (128 B), satisfying the 16-B rule.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// 4-D tiled store shared -> global (same coordinate convention and 128-B
// swizzled shared layout as tma_load_4d), tracked as one bulk async-group.
// The caller issues only non-negative, 16-B aligned coordinates.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 4-D tiled reduce-add shared -> global: the box is added element-wise into
// the tensor (fp32 maps: the fp32 accumulators), performed atomically in L2.
// Same coordinate rules as tma_store_4d; tracked as one bulk async-group.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* smem_src,
                                                  int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group"
      " [%0, {%2, %3, %4, %5}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Order this thread's generic shared-memory accesses before later async-proxy
// (TMA / bulk copy) accesses to the same bytes, e.g. before a buffer that was
// read with ordinary loads is handed back to a bulk-copy producer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Untiled bulk copy global -> shared (both addresses 16-B aligned, size a
// multiple of 16 bytes), completing on an mbarrier transaction count.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk copy shared -> global (both addresses 16-B aligned, size a multiple of
// 16 bytes), tracked per issuing thread as one bulk async-group.
// 64 bytes of one row to global memory: two 32-B stores when the address is
// 32-B aligned (whole sectors, half the store instructions of a warp writing
// 32 rows), else four 16-B stores.
__device__ __forceinline__ void st_global_64B(void* dst, const uint32_t (&w)[16]) {
  if ((reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(w[0]),
                 "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
    asm volatile("st.global.v8.b32 [%0+32], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                 "r"(w[8]), "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]),
                 "r"(w[15])
                 : "memory");
  } else {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(gdst)),
               "r"(smem_addr(ssrc)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until this thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until this thread's bulk stores are complete (writes performed).
__device__ __forceinline__ void bulk_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ------------------------------------------------------------------------------------
// UMMA descriptors
// ------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-B swizzle, sm100 version bits.
//   K-major : lbo ignored (16), sbo = 1024 (stride of 8-row groups)
//   MN-major: lbo = byte stride between 64-element MN blocks, sbo = 1024
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version (Blackwell)
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16 with BF16 A/B, FP32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, fences
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// MMAs and commits are issued by a converged warp: elect.sync picks one lane
// inside the asm block, so the issuing loop stays warp-uniform (operands in
// uniform registers; see mbar_wait for the measured issue rates).
// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void umma_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void umma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every MMA previously issued by this warp completes.
__device__ __forceinline__ void umma_commit_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_addr(bar))
      : "memory");
}

// Pair (cta_group::2) forms.  A kernel uses either these or the cta_group::1
// forms above for all of its tcgen05 allocation, MMA and commit operations.
// Allocation and release are issued by the same warp of both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// M = 256 across the pair (issued by the leader's converged MMA warp): each
// CTA's shared memory holds its 128 rows of A at the A descriptor's address and
// half of B's N columns at the B descriptor's address; each CTA's TMEM receives
// its 128 rows of D at `d_tmem`.
__device__ __forceinline__ void umma_ss_pair_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` in both CTAs of the pair when every pair MMA previously
// issued by this warp completes (the leader: one commit on its own barrier,
// one on the peer CTA's copy through its shared::cluster address).
__device__ __forceinline__ void umma_commit_pair_both_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%1];\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(mapa_shared(bar, 1))
      : "memory");
}

// ------------------------------------------------------------------------------------
// TMEM <-> registers (32 lanes x 32-bit pattern; warp w of a warpgroup owns lanes 32w..)
// ------------------------------------------------------------------------------------
#define G4_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                 "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define G4_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), \
                 "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// Load 32 consecutive columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : G4_R8(0), G4_R8(8), G4_R8(16), G4_R8(24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Make register values produced by tmem_ld32 depend on the wait (keeps the
// compiler from consuming them before tcgen05.wait::ld).
__device__ __forceinline__ void reg_fence32(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}
// Load 16 consecutive columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : G4_R8(0), G4_R8(8)
      : "r"(taddr));
}
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i]));
}
// Store 32 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      G4_W8(0), G4_W8(8), G4_W8(16), G4_W8(24)
      : "memory");
}
// Store 16 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      G4_W8(0), G4_W8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

#undef G4_R8
#undef G4_W8

// ------------------------------------------------------------------------------------
// small numeric helpers
// ------------------------------------------------------------------------------------
constexpr float kLog2e = 1.4426950408889634f;
// Online softmax keeps a stale running max until a tile's max exceeds it by
// more than this many powers of two, so P (bf16, whose relative precision does
// not depend on magnitude) stays below 2^80 and an fp32 row sum or O element
// stays below 2^80 * 2^18 keys * max|V| -- inside fp32 range for |V| < 2^29
// (Gemma-4 values are RMS-normalised).  A rescale drains the MMA pipeline
// (and, in the two-pass forward, rescales a whole 128 x 512 accumulator), so
// the threshold is set where rescales become rare: with unit-RMS d512 vectors
// the score spread is ~30 log2 units and 82% of the causal key tiles of a
// 4096-token sequence would rescale at a threshold of 32, 0.8% at 80.
constexpr float kLazyRescaleLog2 = 80.f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace g4
