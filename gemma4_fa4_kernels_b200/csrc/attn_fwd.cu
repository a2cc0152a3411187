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
  const int lane = tid & 31;
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
  auto ktile = [&](int j) { return klist ? (klist[j] & 0x7fffffff) : kt_lo + j; };
  auto kfull = [&](int j) { return klist != nullptr && (klist[j] & 0x80000000) != 0; };
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
      int* kvis = reinterpret_cast<int*>(misc->xbuf[(j + 1) & 1]);
      int* kdoc = kvis + kTileN;
      if (meta) {
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
      if (cls != 1 && !meta) {
        // text only: the row's visible keys are one range (window bound,
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
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
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
