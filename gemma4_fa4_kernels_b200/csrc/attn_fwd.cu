// Gemma-4 attention forward for sm_100a: TMA-staged Q/K/V tiles feeding
// tcgen05 MMAs with S/P and O accumulators in tensor memory.
//
// One CTA owns a 128-row query tile of one query head and one 256-wide slab
// of the value/output head dimension (local d256: one slab; global d512: two
// slabs, each recomputing the 512-deep QK^T because a 128x512 fp32 O would
// fill all of TMEM).  Warp roles (320 threads):
//   warps 0-7  softmax + epilogue: warps w and w+4 share TMEM lanes
//              32*(w%4).. (their query rows); warp w handles keys [0, 64) of
//              each tile and O columns [0, 128), warp w+4 keys [64, 128) and
//              O columns [128, 256).  The two halves of a row exchange their
//              partial row max through shared memory, so both take identical
//              rescale decisions, and add their row sums at the end.
//   warp  8    TMA producer (one elected lane); also allocates TMEM
//   warp  9    MMA issuer (one elected lane)
// TMEM columns: S0 [0,128), S1 [128,256), O [256,512); P (bf16 pairs) is
// written over the first 64 columns of its S buffer and consumed from TMEM by
// the PV MMA.  K/V chunks stream through a ring of 32 KB shared stages in the
// exact order the MMA warp consumes them: K(0), K(1), V(0), K(2), V(1), ...
//
// Online softmax in the exp2 domain with lazy rescaling: the running max only
// moves (and O is only rescaled) when a tile's max exceeds it by more than
// kLazyRescaleLog2, so P <= 2^kLazyRescaleLog2.  Fully masked rows give O = 0 and LSE = -inf (reference.py:70-75).
//
// Reference interface replaced: flash_attn.cute.flash_attn_func /
// flash_attn_varlen_func forward as called by src/gemma4_fa4/h100.py:766-778,
// 800-815, 864-910, 1013-1036, 1174-1190, 1356-1377.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "g4_attn.cuh"
#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

constexpr int kFwdSoftWarps = 8;
constexpr int kFwdSoftThreads = kFwdSoftWarps * 32;
constexpr int kFwdProducerWarp = kFwdSoftWarps;
constexpr int kFwdMmaWarp = kFwdSoftWarps + 1;
constexpr int kFwdThreads = kFwdSoftThreads + 64;

template <int DQK>
struct FwdCfg {
  static constexpr int kQBytes = DQK * kTileM * 2;
  static constexpr int kStageBytes = 32768;
  static constexpr int kStages = DQK == 256 ? 5 : 3;
  static constexpr int kKChunks = DQK / 128;  // 128-deep K chunks per key tile
  static constexpr int kVChunks = 2;          // 64 keys x 256 values per chunk
  static constexpr int kMiscBytes = 3072;
  static constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + kMiscBytes;
};

struct FwdMisc {
  uint64_t q_full;
  uint64_t ring_full[8];
  uint64_t ring_empty[8];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int k_lo;
  int k_hi;
  int pad[4];
  // Two 1 KB exchange buffers.  Tile j uses xbuf[j & 1] for the partial row
  // maxima ([half][row]) and, with mask metadata, xbuf[(j + 1) & 1] for the
  // tile's key vision / document ids ([0..127] vision, [128..255] document):
  // that buffer's last readers finished before the tile's first barrier.  After
  // the loop xbuf[n_kt & 1] carries the partial row sums.
  float xbuf[2][2 * kTileM];
};
static_assert(sizeof(FwdMisc) <= 3072, "forward misc block exceeds its shared-memory budget");

template <int DQK>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using Cfg = FwdCfg<DQK>;
  extern __shared__ __align__(1024) uint8_t smem[];
  pdl_enter();
  if ((smem_addr(smem) & 1023u) != 0) {  // the 128-B swizzle atoms need 1024-B alignment
    if (p.err) atomicCAS(p.err, 0, 5);
    return;
  }
  uint8_t* q_s = smem;
  uint8_t* ring = smem + Cfg::kQBytes;
  FwdMisc* misc = reinterpret_cast<FwdMisc*>(ring + Cfg::kStages * Cfg::kStageBytes);

  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);  // provably warp-uniform
  // grid (heads, work items, slabs): the head index varies fastest in launch
  // order, so the longest causal rows of every head are dispatched first
  const int head = blockIdx.x;
  const int item = blockIdx.y;
  const int slab = blockIdx.z;
  const int kv_head = head / p.group;

  // ---- work item -> (sequence, query tile) ----
  int seq, qt;
  if (p.tiles != nullptr) {
    if (item >= *p.n_tiles) return;
    const int2 t = p.tiles[item];
    seq = t.x;
    qt = t.y;
  } else {
    const int nqt = (p.layout.seqlen_q + kTileM - 1) / kTileM;
    seq = item % p.layout.batch;
    qt = nqt - 1 - item / p.layout.batch;  // longest causal rows first
  }
  const SeqInfo si = p.layout.seq(seq);
  const int q_off = si.q_off;

  if (tid == 0) {
    mbar_init(&misc->q_full, 1);
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&misc->ring_full[s], 1);
      mbar_init(&misc->ring_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&misc->s_full[b], 1);
      mbar_init(&misc->p_full[b], kFwdSoftThreads);
    }
    mbar_init(&misc->o_done, 1);
    mbar_init(&misc->drain, 1);
    misc->abort = 0;
    misc->k_lo = 0x7fffffff;
    misc->k_hi = -1;
    fence_mbar_init();
  }
  if (warp == kFwdProducerWarp) {
    tmem_alloc(&misc->tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();

  // ---- key range of this query tile (exact bounds; tiles inside are classified) ----
  const int row = tid & (kTileM - 1);  // softmax threads: the TMEM lane (query row)
  const int q_idx = qt * kTileM + row;
  const bool row_valid = tid < kFwdSoftThreads && q_idx < si.len_q;
  const int q_abs = q_idx + q_off;
  int qvis = -1, qdoc = 0;
  if (row_valid) {
    if (p.mask.vis) qvis = p.mask.vis[si.meta_base + q_abs];
    if (p.mask.doc) qdoc = p.mask.doc[si.meta_base + q_abs];
    int lo = p.mask.window > 0 ? max(0, q_abs - p.mask.window + 1) : 0;
    int hi = q_abs;
    if (p.mask.window > 0 && qvis >= 0) {
      hi = p.mask.pair_last ? max(hi, p.mask.pair_last[si.meta_base + q_abs]) : si.len_k - 1;
    }
    if (tid < kTileM) {
      atomicMin(&misc->k_lo, lo);
      atomicMax(&misc->k_hi, min(hi, si.len_k - 1));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = misc->tmem_base;
  // metadata masks: the planner's exact key-tile list of this query tile (each
  // listed tile holds an allowed pair; tiles outside the list are never loaded)
  const int* klist = nullptr;
  int kt_lo, n_kt;
  if (p.klist) {
    const int g = p.tiles ? item : seq * ((p.layout.seqlen_q + kTileM - 1) / kTileM) + qt;
    klist = p.klist + static_cast<int64_t>(g) * p.klist_stride;
    kt_lo = 0;
    n_kt = p.ranges[g].y;
  } else {
    kt_lo = misc->k_hi >= 0 ? misc->k_lo / kTileN : 0;
    n_kt = misc->k_hi >= 0 ? misc->k_hi / kTileN - kt_lo + 1 : 0;
  }
  // key tile of step j, and whether the planner found every pair of it allowed
  auto ktile = [&](int j) { return klist ? (klist[j] & kTileEntryIndex) : kt_lo + j; };
  auto kfull = [&](int j) { return klist != nullptr && (klist[j] & kTileEntryFull) != 0; };
  auto ktext = [&](int j) { return klist != nullptr && (klist[j] & kTileEntryText) != 0; };
  const CtaAbort ab{&misc->abort, p.err};

  if (warp == kFwdProducerWarp) {
    // ============================ TMA producer ============================
    // whole warp: warp-uniform waits, copies issued by one elected lane
    if (n_kt > 0) {
      if (elect_one()) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        mbar_expect_tx(&misc->q_full, Cfg::kQBytes);
        for (int blk = 0; blk < DQK / 64; ++blk)
          tma_load_4d(q_s + blk * 16384, &tmQ, &misc->q_full, blk * 64, head,
                      si.q_base + qt * kTileM, si.b_coord);
      }
      __syncwarp();
      uint32_t it = 0;
      bool ok = true;
      auto acquire = [&](uint32_t& stage) -> bool {
        stage = it % Cfg::kStages;
        const uint32_t ph = (it / Cfg::kStages) & 1;
        return mbar_wait(&misc->ring_empty[stage], ph ^ 1, ab, kDevTimeoutMma);
      };
      auto load_k = [&](int kt) {
        for (int c = 0; c < Cfg::kKChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = acquire(st))) break;
          if (elect_one()) {
            mbar_expect_tx(&misc->ring_full[st], Cfg::kStageBytes);
            uint8_t* dst = ring + st * Cfg::kStageBytes;
            for (int h = 0; h < 2; ++h)
              tma_load_4d(dst + h * 16384, &tmK, &misc->ring_full[st], (2 * c + h) * 64, kv_head,
                          si.k_base + kt * kTileN, si.b_coord);
          }
          __syncwarp();
          ++it;
        }
      };
      auto load_v = [&](int kt) {
        for (int c = 0; c < Cfg::kVChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = acquire(st))) break;
          if (elect_one()) {
            mbar_expect_tx(&misc->ring_full[st], Cfg::kStageBytes);
            uint8_t* dst = ring + st * Cfg::kStageBytes;
            for (int blk = 0; blk < 4; ++blk)
              tma_load_4d(dst + blk * 8192, &tmV, &misc->ring_full[st], slab * 256 + blk * 64,
                          kv_head, si.k_base + kt * kTileN + c * 64, si.b_coord);
          }
          __syncwarp();
          ++it;
        }
      };
      load_k(ktile(0));
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt) load_k(ktile(j + 1));
        load_v(ktile(j));
      }
    }
    __syncwarp();
  } else if (warp == kFwdMmaWarp) {
    // ============================ MMA issuer ============================
    // the whole warp runs the issue loop (warp-uniform waits, one elected lane
    // per MMA): see mbar_wait
    if (n_kt > 0) {
      constexpr uint32_t kIdS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdPV = idesc_bf16(128, 256, false, true);
      const uint32_t q_base = smem_addr(q_s);
      const uint32_t ring_base = smem_addr(ring);
      uint32_t it = 0;
      bool ok = mbar_wait(&misc->q_full, 0, ab, kDevTimeoutTma);
      auto take = [&](uint32_t& stage) -> bool {
        stage = it % Cfg::kStages;
        const uint32_t ph = (it / Cfg::kStages) & 1;
        if (!mbar_wait(&misc->ring_full[stage], ph, ab, kDevTimeoutTma)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int j) {
        const uint32_t d = tmem + (j & 1) * 128;
        for (int c = 0; c < Cfg::kKChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = take(st))) break;
          const uint32_t kb = ring_base + st * Cfg::kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int g = c * 8 + kk;
            const uint64_t a = sdesc_sw128(q_base + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024);
            const uint64_t b = sdesc_sw128(kb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            umma_ss_w(d, a, b, kIdS, (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
          ++it;
        }
        umma_commit_w(&misc->s_full[j & 1]);
      };
      auto issue_pv = [&](int j) {
        const uint32_t a_t = tmem + (j & 1) * 128;
        for (int c = 0; c < Cfg::kVChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = take(st))) break;
          const uint32_t vb = ring_base + st * Cfg::kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t b = sdesc_sw128(vb + kk * 2048, 8192, 1024);
            umma_ts_w(tmem + 256, a_t + c * 32 + kk * 8, b, kIdPV, (j | c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
          ++it;
        }
        umma_commit_w(&misc->o_done);
      };
      if (ok) issue_s(0);
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt) issue_s(j + 1);
        if (!(ok = mbar_wait(&misc->p_full[j & 1], (j >> 1) & 1, ab, kDevTimeoutPeer)))
          break;
        tc_fence_after();
        issue_pv(j);
      }
      // Drain: every MMA this warp issued has completed before TMEM is freed.
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ======================= softmax + epilogue (warps 0-7) =======================
    // Every tcgen05.ld/st below is .sync.aligned, so all control flow around
    // them is kept warp-uniform: `ok` is reduced with __all_sync after each
    // wait and the rescale decision with __any_sync.  Loops never break, and
    // the named barrier 1 (all softmax threads) is reached once per tile (twice
    // with mask metadata) by every thread, whatever `ok` says.
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int half = warp >> 2;  // keys [64*half, +64) of a tile; O columns [128*half, +128)
    const bool meta = p.mask.has_meta();
    const int qa0 = qt * kTileM + q_off;
    const int qa1 = min((qt + 1) * kTileM, si.len_q) - 1 + q_off;
    float m_run = -INFINITY;  // running max, log2 domain
    float l_half = 0.f;       // this half's share of the row sum
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int k0 = ktile(j) * kTileN;
      const int kh = k0 + half * 64;  // first key of this thread's half
      const int cls = klist ? (kfull(j) ? 1 : 2)
                            : (meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0, si.len_k));
      const bool text_rule = !meta || ktext(j);
      int* kvis = reinterpret_cast<int*>(misc->xbuf[(j + 1) & 1]);
      int* kdoc = kvis + kTileN;
      if (!text_rule) {
        asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
        if (tid < kTileN) {
          const int kk = k0 + tid;
          const bool in = kk < si.len_k;
          kvis[tid] = (p.mask.vis && in) ? p.mask.vis[si.meta_base + kk] : -1;
          kdoc[tid] = (p.mask.doc && in) ? p.mask.doc[si.meta_base + kk] : 0;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
      }
      if (ok) ok = mbar_wait(&misc->s_full[j & 1], (j >> 1) & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      float s[64];
      if (ok) {
        tc_fence_after();
        uint32_t r0[32], r1[32];
        const uint32_t sb = lane_base + (j & 1) * 128 + half * 64;
        tmem_ld32(sb + 0, r0);
        tmem_ld32(sb + 32, r1);
        tmem_wait_ld();
        reg_fence32(r0);
        reg_fence32(r1);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = -INFINITY;
      }
      if (cls != 1 && text_rule) {
        // text rule: the row's visible keys are one range (window bound,
        // causal bound, end of the sequence)
        const int k_lo = p.mask.window > 0 ? q_abs - p.mask.window + 1 : 0;
        const int k_hi = min(q_abs, si.len_k - 1);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (kh + i < k_lo || kh + i > k_hi) s[i] = -INFINITY;
      } else if (cls != 1) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int k = kh + i;
          const bool keep = k < si.len_k &&
                            mask_allows(p.mask.window, q_abs, k, qvis, qdoc, kvis[half * 64 + i],
                                        kdoc[half * 64 + i]);
          if (!keep) s[i] = -INFINITY;
        }
      }
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) mt = fmaxf(mt, s[i]);
      float* pm = misc->xbuf[j & 1];
      pm[half * kTileM + row] = mt * kLog2e;
      asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
      mt = fmaxf(pm[row], pm[kTileM + row]);
      float alpha = 1.f;
      bool rescale = false;
      if (mt > m_run + kLazyRescaleLog2) {  // also true for the first finite tile
        // a row without any finite score so far has O = 0 and l = 0: no correction
        if (m_run != -INFINITY) {
          alpha = ex2(m_run - mt);
          rescale = true;
        }
        m_run = mt;
      }
      if (!ok) continue;
      const float m_sub = (m_run == -INFINITY) ? 0.f : m_run;
      float rowsum = 0.f;
      {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2(fmaf(s[2 * i], kLog2e, -m_sub));
          const float p1 = ex2(fmaf(s[2 * i + 1], kLog2e, -m_sub));
          rowsum += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        // P (bf16 pairs) over the first 64 columns of the S buffer: keys
        // [64*half, +64) at columns [32*half, +32)
        tmem_st32(lane_base + (j & 1) * 128 + half * 32, pk);
      }
      l_half = l_half * alpha + rowsum;
      tmem_wait_st();
      if (j > 0) {
        ok = mbar_wait(&misc->o_done, (j - 1) & 1, ab, kDevTimeoutMma);
        ok = __all_sync(0xffffffffu, ok);
        if (ok && __any_sync(0xffffffffu, rescale)) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; c += 2) {
            const uint32_t oc = lane_base + 256 + half * 128 + c * 32;
            uint32_t r0[32], r1[32];
            tmem_ld32(oc, r0);
            tmem_ld32(oc + 32, r1);
            tmem_wait_ld();
            reg_fence32(r0);
            reg_fence32(r1);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              r0[i] = __float_as_uint(__uint_as_float(r0[i]) * alpha);
              r1[i] = __float_as_uint(__uint_as_float(r1[i]) * alpha);
            }
            tmem_st32(oc, r0);
            tmem_st32(oc + 32, r1);
          }
          tmem_wait_st();
        }
      }
      tc_fence_before();
      if (ok) mbar_arrive(&misc->p_full[j & 1]);
    }
    // ---- epilogue: O / l -> bf16, LSE ----
    float* ls = misc->xbuf[n_kt & 1];
    ls[half * kTileM + row] = l_half;
    asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
    const float l_run = ls[row] + ls[kTileM + row];
    if (ok && n_kt > 0) ok = mbar_wait(&misc->o_done, (n_kt - 1) & 1, ab, kDevTimeoutMma);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool have_o = ok && n_kt > 0;
    const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
    __nv_bfloat16* orow = p.o + static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
                          static_cast<int64_t>(si.q_base + q_idx) * p.o_stride[1] +
                          static_cast<int64_t>(head) * p.o_stride[2] + slab * 256 + half * 128;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      if (have_o) {
        tmem_ld32(lane_base + 256 + half * 128 + c * 32, r);
        tmem_wait_ld();
        reg_fence32(r);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (row_valid) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv_l,
                              __uint_as_float(r[2 * i + 1]) * inv_l);
        st_global_64B(orow + c * 32, pk);
      }
    }
    if (row_valid && slab == 0 && half == 0) {
      const float lse = (l_run > 0.f) ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
      p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
            static_cast<int64_t>(head) * p.lse_stride[1] + si.q_base + q_idx] = lse;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFwdProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// Persistent local forward (d256).  Local layers give every query tile at most
// nine or ten key tiles, so a CTA's start (barrier set-up, TMEM allocation, the
// resident Q load, the first S) and end (the O epilogue) are a large share of a
// one-tile CTA's life.  Here one CTA per SM walks the (head, query tile) items in
// the same longest-first order (round i of CTA c takes item i * G + c, or
// i * G + G - 1 - c in odd rounds, for G CTAs), and the
// roles run ahead across items: the producer loads the next item's Q as soon as
// the current item's last S MMA has read Q (q_free) and streams its K/V into the
// same ring; the MMA warp issues the next item's first S while the softmax
// warps write the current item's O, and its first PV (which overwrites O) waits
// until they have read it (o_free).  Barrier phases follow global counters:
// tiles T over all items (S/P buffers, o_done) and active items I (q_full,
// q_free, o_free).
// =====================================================================================
struct FwdItem {
  bool valid;   // an item of the problem
  int head, seq, qt, g;
  SeqInfo si;
  int kt_lo, n_kt;
  const int* klist;
};

__device__ __forceinline__ FwdItem fwd_item(const FwdParams& p, int64_t L, int num_q_heads) {
  FwdItem it;
  it.valid = false;
  it.n_kt = 0;
  it.kt_lo = 0;
  it.klist = nullptr;
  const int nqt = (p.layout.seqlen_q + kTileM - 1) / kTileM;
  const int64_t items = static_cast<int64_t>(num_q_heads) *
                        (p.tiles != nullptr ? int64_t(*p.n_tiles) : int64_t(p.layout.batch) * nqt);
  if (L >= items) return it;
  it.head = static_cast<int>(L % num_q_heads);
  const int item = static_cast<int>(L / num_q_heads);
  if (p.tiles != nullptr) {
    const int2 t = p.tiles[item];
    it.seq = t.x;
    it.qt = t.y;
    it.g = item;
  } else {
    it.seq = item % p.layout.batch;
    it.qt = nqt - 1 - item / p.layout.batch;  // longest causal rows first
    it.g = it.seq * nqt + it.qt;
  }
  it.si = p.layout.seq(it.seq);
  it.valid = true;
  if (p.klist) {
    it.klist = p.klist + static_cast<int64_t>(it.g) * p.klist_stride;
    it.n_kt = p.ranges[it.g].y;
  } else {
    const int qa0 = it.qt * kTileM + it.si.q_off;
    const int qa1 = min((it.qt + 1) * kTileM, it.si.len_q) - 1 + it.si.q_off;
    const int lo = p.mask.window > 0 ? max(0, qa0 - p.mask.window + 1) : 0;
    const int hi = min(qa1, it.si.len_k - 1);
    if (hi >= lo) {
      it.kt_lo = lo / kTileN;
      it.n_kt = hi / kTileN - it.kt_lo + 1;
    }
  }
  return it;
}
// Item of round i for this CTA: rounds alternate direction (CTA c takes items
// c, 2G-1-c, 2G+c, ...), which evens out the longest-first costs per CTA.
__device__ __forceinline__ int64_t fwd_item_index(int64_t i) {
  const int64_t g = gridDim.x;
  return i * g + ((i & 1) ? g - 1 - blockIdx.x : blockIdx.x);
}
__device__ __forceinline__ int fwd_ktile(const FwdItem& it, int j) {
  return it.klist ? (it.klist[j] & kTileEntryIndex) : it.kt_lo + j;
}

// Four more warps write each item's O: the softmax warps hand over the row
// normalisers and go on with the next item while O leaves TMEM (the next
// item's first P V, which overwrites O, waits for them through o_free).
constexpr int kFwdPThreads = kFwdThreads + 128;  // warps 10-13

struct FwdPMisc {
  uint64_t q_full;
  uint64_t q_free;
  uint64_t o_free;
  uint64_t epi_full;          // the softmax warps wrote an item's 1/l (256 arrivals)
  uint64_t epi_empty;         // the epilogue warps read it (128 arrivals)
  uint64_t ring_full[8];
  uint64_t ring_empty[8];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done[2];         // P V of tile t complete (o_done[t & 1], phase t >> 1)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float xbuf[2][2 * kTileM];  // as FwdMisc::xbuf, indexed by the global tile parity
  float inv_l[kTileM];        // the current item's 1 / rowsum, for the epilogue warps
};
static_assert(sizeof(FwdPMisc) <= 3072, "persistent forward misc block exceeds its budget");

__global__ void __launch_bounds__(kFwdPThreads, 1)
    attn_fwd_persistent_kernel(const __grid_constant__ CUtensorMap tmQ,
                               const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const FwdParams p,
                               int num_q_heads) {
  constexpr int DQK = 256;
  using Cfg = FwdCfg<DQK>;
  extern __shared__ __align__(1024) uint8_t smem[];
  pdl_enter();
  if ((smem_addr(smem) & 1023u) != 0) {
    if (p.err) atomicCAS(p.err, 0, 5);
    return;
  }
  uint8_t* q_s = smem;
  uint8_t* ring = smem + Cfg::kQBytes;
  FwdPMisc* misc = reinterpret_cast<FwdPMisc*>(ring + Cfg::kStages * Cfg::kStageBytes);
  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);

  if (tid == 0) {
    mbar_init(&misc->q_full, 1);
    mbar_init(&misc->q_free, 1);
    mbar_init(&misc->o_free, 128);  // the epilogue warps
    mbar_init(&misc->epi_full, kFwdSoftThreads);
    mbar_init(&misc->epi_empty, 128);
    for (int s2 = 0; s2 < Cfg::kStages; ++s2) {
      mbar_init(&misc->ring_full[s2], 1);
      mbar_init(&misc->ring_empty[s2], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&misc->s_full[b], 1);
      mbar_init(&misc->p_full[b], kFwdSoftThreads);
    }
    mbar_init(&misc->o_done[0], 1);
    mbar_init(&misc->o_done[1], 1);
    mbar_init(&misc->drain, 1);
    misc->abort = 0;
    fence_mbar_init();
  }
  if (warp == kFwdProducerWarp) {
    tmem_alloc(&misc->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;
  const CtaAbort ab{&misc->abort, p.err};

  if (warp == kFwdProducerWarp) {
    // ============================ TMA producer ============================
    uint32_t it = 0;   // ring slots used so far
    int I = 0;         // active items so far
    bool ok = true;
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
    }
    __syncwarp();
    auto acquire = [&](uint32_t& stage) -> bool {
      stage = it % Cfg::kStages;
      const uint32_t ph = (it / Cfg::kStages) & 1;
      return mbar_wait(&misc->ring_empty[stage], ph ^ 1, ab, kDevTimeoutMma);
    };
    // K / V chunks in the MMA warp's order: K of tile t + 1 before V of tile
    // t, across items too (the next item's first K goes before the current
    // item's last V, which is held back until then)
    auto load_k = [&](const FwdItem& w, int kt) {
      const int kv_head = w.head / p.group;
      for (int c = 0; c < Cfg::kKChunks && ok; ++c) {
        uint32_t st;
        if (!(ok = acquire(st))) break;
        if (elect_one()) {
          mbar_expect_tx(&misc->ring_full[st], Cfg::kStageBytes);
          uint8_t* dst = ring + st * Cfg::kStageBytes;
          for (int h = 0; h < 2; ++h)
            tma_load_4d(dst + h * 16384, &tmK, &misc->ring_full[st], (2 * c + h) * 64, kv_head,
                        w.si.k_base + kt * kTileN, w.si.b_coord);
        }
        __syncwarp();
        ++it;
      }
    };
    auto load_v = [&](const FwdItem& w, int kt) {
      const int kv_head = w.head / p.group;
      for (int c = 0; c < Cfg::kVChunks && ok; ++c) {
        uint32_t st;
        if (!(ok = acquire(st))) break;
        if (elect_one()) {
          mbar_expect_tx(&misc->ring_full[st], Cfg::kStageBytes);
          uint8_t* dst = ring + st * Cfg::kStageBytes;
          for (int blk = 0; blk < 4; ++blk)
            tma_load_4d(dst + blk * 8192, &tmV, &misc->ring_full[st], blk * 64, kv_head,
                        w.si.k_base + kt * kTileN + c * 64, w.si.b_coord);
        }
        __syncwarp();
        ++it;
      }
    };
    FwdItem held;  // the item whose last V tile is held back
    int held_kt = -1;
    for (int64_t i = 0; ok; ++i) {
      const FwdItem wi = fwd_item(p, fwd_item_index(i), num_q_heads);
      if (!wi.valid) break;
      if (wi.n_kt == 0) continue;
      // Q of this item once the previous item's S MMAs have read the last one
      if (I > 0 && !(ok = mbar_wait(&misc->q_free, (I - 1) & 1, ab, kDevTimeoutMma))) break;
      if (elect_one()) {
        mbar_expect_tx(&misc->q_full, Cfg::kQBytes);
        for (int blk = 0; blk < DQK / 64; ++blk)
          tma_load_4d(q_s + blk * 16384, &tmQ, &misc->q_full, blk * 64, wi.head,
                      wi.si.q_base + wi.qt * kTileM, wi.si.b_coord);
      }
      __syncwarp();
      load_k(wi, fwd_ktile(wi, 0));
      if (held_kt >= 0) load_v(held, held_kt);
      for (int j = 0; j < wi.n_kt && ok; ++j) {
        if (j + 1 < wi.n_kt) {
          load_k(wi, fwd_ktile(wi, j + 1));
          load_v(wi, fwd_ktile(wi, j));
        } else {
          held = wi;
          held_kt = fwd_ktile(wi, j);
        }
      }
      ++I;
    }
    if (held_kt >= 0 && ok) load_v(held, held_kt);
    __syncwarp();
  } else if (warp == kFwdMmaWarp) {
    // ============================ MMA issuer ============================
    constexpr uint32_t kIdS = idesc_bf16(128, 128, false, false);
    constexpr uint32_t kIdPV = idesc_bf16(128, 256, false, true);
    const uint32_t q_base = smem_addr(q_s);
    const uint32_t ring_base = smem_addr(ring);
    uint32_t it = 0;
    int64_t T = 0;  // tiles so far (all items)
    int I = 0;
    bool ok = true;
    auto take = [&](uint32_t& stage) -> bool {
      stage = it % Cfg::kStages;
      const uint32_t ph = (it / Cfg::kStages) & 1;
      if (!mbar_wait(&misc->ring_full[stage], ph, ab, kDevTimeoutTma)) return false;
      tc_fence_after();
      return true;
    };
    auto issue_s = [&](int64_t t) {
      const uint32_t d = tmem + static_cast<uint32_t>(t & 1) * 128;
      for (int c = 0; c < Cfg::kKChunks && ok; ++c) {
        uint32_t st;
        if (!(ok = take(st))) break;
        const uint32_t kb = ring_base + st * Cfg::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int g = c * 8 + kk;
          const uint64_t a = sdesc_sw128(q_base + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024);
          const uint64_t b = sdesc_sw128(kb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          umma_ss_w(d, a, b, kIdS, (c | kk) != 0);
        }
        umma_commit_w(&misc->ring_empty[st]);
        ++it;
      }
      umma_commit_w(&misc->s_full[t & 1]);
    };
    auto issue_pv = [&](int64_t t, bool first) {
      const uint32_t a_t = tmem + static_cast<uint32_t>(t & 1) * 128;
      for (int c = 0; c < Cfg::kVChunks && ok; ++c) {
        uint32_t st;
        if (!(ok = take(st))) break;
        const uint32_t vb = ring_base + st * Cfg::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t b = sdesc_sw128(vb + kk * 2048, 8192, 1024);
          umma_ts_w(tmem + 256, a_t + c * 32 + kk * 8, b, kIdPV, !(first && c == 0 && kk == 0));
        }
        umma_commit_w(&misc->ring_empty[st]);
        ++it;
      }
      umma_commit_w(&misc->o_done[t & 1]);
    };
    // Items with key tiles, in order; the next item's first S is issued before
    // the current item's last P V (it waits only for the next Q), so the
    // softmax warps find it ready when they finish an item.
    int64_t cursor = 0;
    auto next_item = [&]() {
      for (;; ++cursor) {
        const FwdItem w = fwd_item(p, fwd_item_index(cursor), num_q_heads);
        if (!w.valid || w.n_kt > 0) {
          ++cursor;
          return w;
        }
      }
    };
    FwdItem cur = next_item();
    if (cur.valid) {
      if ((ok = mbar_wait(&misc->q_full, 0, ab, kDevTimeoutTma))) {
        tc_fence_after();
        issue_s(0);
        if (cur.n_kt == 1) umma_commit_w(&misc->q_free);
      }
    }
    while (cur.valid && ok) {
      const int n = cur.n_kt;
      const FwdItem nxt = next_item();
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) {
          issue_s(T + j + 1);
          if (j + 2 == n) umma_commit_w(&misc->q_free);  // the item's last S: Q may be replaced
        } else if (nxt.valid) {
          if (!(ok = mbar_wait(&misc->q_full, (I + 1) & 1, ab, kDevTimeoutTma))) break;
          tc_fence_after();
          issue_s(T + n);
          if (nxt.n_kt == 1) umma_commit_w(&misc->q_free);
        }
        const int64_t t = T + j;
        if (!(ok = mbar_wait(&misc->p_full[t & 1], (t >> 1) & 1, ab, kDevTimeoutPeer))) break;
        if (j == 0 && I > 0 &&
            !(ok = mbar_wait(&misc->o_free, (I - 1) & 1, ab, kDevTimeoutPeer)))
          break;
        tc_fence_after();
        issue_pv(t, j == 0);
      }
      T += n;
      ++I;
      cur = nxt;
    }
    umma_commit_w(&misc->drain);
    mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    __syncwarp();
  } else if (warp < kFwdSoftWarps) {
    // ======================= softmax (warps 0-7) =======================
    // Control flow stays uniform over the 256 softmax threads: every item and
    // tile reaches named barrier 1 the same number of times whatever `ok` says.
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int half = warp >> 2;
    const int row = tid & (kTileM - 1);
    const bool meta = p.mask.has_meta();
    bool ok = true;
    int64_t T = 0;
    int I = 0;
    for (int64_t i = 0;; ++i) {
      const FwdItem wi = fwd_item(p, fwd_item_index(i), num_q_heads);
      if (!wi.valid) break;
      const SeqInfo& si = wi.si;
      const int q_off = si.q_off;
      const int q_idx = wi.qt * kTileM + row;
      const bool row_valid = q_idx < si.len_q;
      const int q_abs = q_idx + q_off;
      const int qvis = (row_valid && p.mask.vis) ? p.mask.vis[si.meta_base + q_abs] : -1;
      const int qdoc = (row_valid && p.mask.doc) ? p.mask.doc[si.meta_base + q_abs] : 0;
      // Metadata masks read a list entry and, for tiles that are not full, the
      // keys' vision / document ids: both are loaded ahead (the entry two tiles,
      // the ids one tile before use) so their latency hides under the softmax.
      // Entries are bounded by the row's capacity, not its length, so the first
      // two are requested together with the length; entries past it go unused.
      auto entry = [&](int j) { return (wi.klist && j < p.klist_stride) ? wi.klist[j] : 0; };
      int ent_cur = entry(0), ent_nxt = entry(1);
      const int qa0 = wi.qt * kTileM + q_off;
      const int qa1 = min((wi.qt + 1) * kTileM, si.len_q) - 1 + q_off;
      const int n = wi.n_kt;
      __nv_bfloat16* orow = p.o + static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
                            static_cast<int64_t>(si.q_base + q_idx) * p.o_stride[1] +
                            static_cast<int64_t>(wi.head) * p.o_stride[2] + half * 128;
      float* lse_row = p.lse + static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
                       static_cast<int64_t>(wi.head) * p.lse_stride[1] + si.q_base + q_idx;
      if (n == 0) {  // no visible key: O = 0, LSE = -inf
        if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
          for (int i = 0; i < 16; ++i) dst[i] = make_uint4(0, 0, 0, 0);
          if (half == 0) *lse_row = -INFINITY;
        }
        continue;
      }
      float m_run = -INFINITY, l_half = 0.f;
      auto key_meta = [&](int ent, int j, int& mv, int& md) {
        mv = -1;
        md = 0;
        if (!meta || tid >= kTileN || j >= n ||
            (wi.klist && (ent & (kTileEntryFull | kTileEntryText))))
          return;
        const int kk = (wi.klist ? (ent & kTileEntryIndex) : wi.kt_lo + j) * kTileN + tid;
        if (kk < si.len_k) {
          if (p.mask.vis) mv = p.mask.vis[si.meta_base + kk];
          if (p.mask.doc) md = p.mask.doc[si.meta_base + kk];
        }
      };
      int mv_cur, md_cur;
      key_meta(ent_cur, 0, mv_cur, md_cur);
      for (int j = 0; j < n; ++j) {
        const int64_t t = T + j;
        const int ent = ent_cur;
        const int ent2 = entry(j + 2);
        int mv_nxt, md_nxt;
        key_meta(ent_nxt, j + 1, mv_nxt, md_nxt);
        const int k0 = (wi.klist ? (ent & kTileEntryIndex) : wi.kt_lo + j) * kTileN;
        const int kh = k0 + half * 64;
        const bool text_rule = !meta || (wi.klist && (ent & kTileEntryText));
        const int cls = wi.klist ? ((ent & kTileEntryFull) ? 1 : 2)
                                 : (meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0,
                                                               si.len_k));
        int* kvis = reinterpret_cast<int*>(misc->xbuf[(t + 1) & 1]);
        int* kdoc = kvis + kTileN;
        if (!text_rule && cls != 1) {  // the same for all 256 threads
          asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
          if (tid < kTileN) {
            kvis[tid] = mv_cur;
            kdoc[tid] = md_cur;
          }
          asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
        }
        ent_cur = ent_nxt;
        ent_nxt = ent2;
        mv_cur = mv_nxt;
        md_cur = md_nxt;
        if (ok) ok = mbar_wait(&misc->s_full[t & 1], (t >> 1) & 1, ab, kDevTimeoutMma);
        ok = __all_sync(0xffffffffu, ok);
        float sv[64];
        if (ok) {
          tc_fence_after();
          uint32_t r0[32], r1[32];
          const uint32_t sb = lane_base + static_cast<uint32_t>(t & 1) * 128 + half * 64;
          tmem_ld32(sb + 0, r0);
          tmem_ld32(sb + 32, r1);
          tmem_wait_ld();
          reg_fence32(r0);
          reg_fence32(r1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            sv[i] = __uint_as_float(r0[i]);
            sv[32 + i] = __uint_as_float(r1[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) sv[i] = -INFINITY;
        }
        if (cls != 1 && text_rule) {
          const int k_lo = p.mask.window > 0 ? q_abs - p.mask.window + 1 : 0;
          const int k_hi = min(q_abs, si.len_k - 1);
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kh + i < k_lo || kh + i > k_hi) sv[i] = -INFINITY;
        } else if (cls != 1) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int k = kh + i;
            const bool keep = k < si.len_k &&
                              mask_allows(p.mask.window, q_abs, k, qvis, qdoc,
                                          kvis[half * 64 + i], kdoc[half * 64 + i]);
            if (!keep) sv[i] = -INFINITY;
          }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) mt = fmaxf(mt, sv[i]);
        float* pm = misc->xbuf[t & 1];
        pm[half * kTileM + row] = mt * kLog2e;
        asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
        mt = fmaxf(pm[row], pm[kTileM + row]);
        float alpha = 1.f;
        bool rescale = false;
        if (mt > m_run + kLazyRescaleLog2) {
          if (m_run != -INFINITY) {
            alpha = ex2(m_run - mt);
            rescale = true;
          }
          m_run = mt;
        }
        if (!ok) continue;
        const float m_sub = (m_run == -INFINITY) ? 0.f : m_run;
        float rowsum = 0.f;
        {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float p0 = ex2(fmaf(sv[2 * i], kLog2e, -m_sub));
            const float p1 = ex2(fmaf(sv[2 * i + 1], kLog2e, -m_sub));
            rowsum += p0 + p1;
            pk[i] = pack_bf16x2(p0, p1);
          }
          tmem_st32(lane_base + static_cast<uint32_t>(t & 1) * 128 + half * 32, pk);
        }
        l_half = l_half * alpha + rowsum;
        tmem_wait_st();
        // a warp that rescales O waits for the previous tile's P V first; the
        // others hand P over at once (P V of tile t - 1 reads the other buffer).
        // With a barrier per tile parity, no wait is ever two phases behind.
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          if (ok) ok = mbar_wait(&misc->o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, ab, kDevTimeoutMma);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 4; c += 2) {
              const uint32_t oc = lane_base + 256 + half * 128 + c * 32;
              uint32_t r0[32], r1[32];
              tmem_ld32(oc, r0);
              tmem_ld32(oc + 32, r1);
              tmem_wait_ld();
              reg_fence32(r0);
              reg_fence32(r1);
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                r0[i] = __float_as_uint(__uint_as_float(r0[i]) * alpha);
                r1[i] = __float_as_uint(__uint_as_float(r1[i]) * alpha);
              }
              tmem_st32(oc, r0);
              tmem_st32(oc + 32, r1);
            }
            tmem_wait_st();
          }
        }
        tc_fence_before();
        if (ok) mbar_arrive(&misc->p_full[t & 1]);
      }
      // ---- item end: LSE, and 1/l for the epilogue warps, which write O ----
      float* ls = misc->xbuf[(T + n) & 1];
      ls[half * kTileM + row] = l_half;
      asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
      const float l_run = ls[row] + ls[kTileM + row];
      // every thread has read the sums before the next item's first tile reuses
      // this buffer for its row maxima
      asm volatile("bar.sync 1, %0;" ::"n"(kFwdSoftThreads) : "memory");
      // the epilogue warps have read the previous item's 1/l
      if (I > 0 && ok) ok = mbar_wait(&misc->epi_empty, (I - 1) & 1, ab, kDevTimeoutPeer);
      ok = __all_sync(0xffffffffu, ok);
      if (half == 0) misc->inv_l[row] = (l_run > 0.f) ? 1.f / l_run : 0.f;
      mbar_arrive(&misc->epi_full);
      if (row_valid && half == 0)
        *lse_row = (l_run > 0.f) ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
      T += n;
      ++I;
    }
  } else {
    // ======================= O epilogue (warps 10-13) =======================
    // Warp w reads TMEM lane quarter w % 4: one row per thread, all 256
    // columns, normalised by the softmax warps' 1/l and stored to O; then O is
    // free for the next item's first P V.
    const int q4 = warp & 3;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int row = q4 * 32 + (tid & 31);
    bool ok = true;
    int64_t T = 0;
    int I = 0;
    for (int64_t i = 0;; ++i) {
      const FwdItem wi = fwd_item(p, fwd_item_index(i), num_q_heads);
      if (!wi.valid) break;
      const int n = wi.n_kt;
      if (n == 0) continue;  // the softmax warps wrote that item's zeros
      const SeqInfo& si = wi.si;
      const int q_idx = wi.qt * kTileM + row;
      const bool row_valid = q_idx < si.len_q;
      __nv_bfloat16* orow = p.o + static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
                            static_cast<int64_t>(si.q_base + q_idx) * p.o_stride[1] +
                            static_cast<int64_t>(wi.head) * p.o_stride[2];
      if (ok) ok = mbar_wait(&misc->epi_full, I & 1, ab, kDevTimeoutPeer);
      ok = __all_sync(0xffffffffu, ok);
      const float inv_l = misc->inv_l[row];
      mbar_arrive(&misc->epi_empty);
      if (ok)
        ok = mbar_wait(&misc->o_done[(T + n - 1) & 1], ((T + n - 1) >> 1) & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 8; c += 2) {
        uint32_t r[2][32];
        if (ok) {
          tmem_ld32(lane_base + 256 + c * 32, r[0]);
          tmem_ld32(lane_base + 256 + c * 32 + 32, r[1]);
          tmem_wait_ld();
          reg_fence32(r[0]);
          reg_fence32(r[1]);
        } else {
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) r[0][i2] = r[1][i2] = 0u;
        }
        if (row_valid) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t pk[16];
#pragma unroll
            for (int i2 = 0; i2 < 16; ++i2)
              pk[i2] = pack_bf16x2(__uint_as_float(r[hh][2 * i2]) * inv_l,
                                   __uint_as_float(r[hh][2 * i2 + 1]) * inv_l);
            st_global_64B(orow + (c + hh) * 32, pk);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&misc->o_free);
      T += n;
      ++I;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFwdProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_fwd_persistent(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const FwdParams& p, int ctas, int num_q_heads, cudaStream_t stream) {
  using Cfg = FwdCfg<256>;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_persistent_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = launch_chained(attn_fwd_persistent_kernel, dim3(ctas), dim3(kFwdPThreads), Cfg::kSmemBytes,
                     stream, tq, tk, tv, p, num_q_heads);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

template <int DQK>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
               const FwdParams& p, int grid_x, int num_q_heads, int slabs, cudaStream_t stream) {
  using Cfg = FwdCfg<DQK>;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<DQK>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = launch_chained(attn_fwd_kernel<DQK>, dim3(num_q_heads, grid_x, slabs), dim3(kFwdThreads),
                     Cfg::kSmemBytes, stream, tq, tk, tv, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

template int launch_fwd<256>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                             const FwdParams&, int, int, int, cudaStream_t);
template int launch_fwd<512>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                             const FwdParams&, int, int, int, cudaStream_t);

}  // namespace g4
