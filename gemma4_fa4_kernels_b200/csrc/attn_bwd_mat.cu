// Gemma-4 attention backward for sm_100a with materialised P / dS tiles.
//
// A 128x512 fp32 accumulator fills all of tensor memory, so a KV-major kernel
// cannot hold dK and dV (or dQ next to S and dP) for d512; splitting their
// columns over CTAs forces every CTA to recompute the 512-deep S = QK^T and
// dP = dO V^T.  This path instead spends HBM (ample on B200) to compute each of
// the five backward matmuls exactly once:
//
//   plan   per query tile: first key tile, key-tile count and the offset of its
//          tiles in the scratch (prefix sum over the causal / window band);
//   score  Q-major.  S = Q K^T and/or dP = dO V^T into double-buffered TMEM;
//          the four math warps write P = exp(S - LSE) and dS = P (dP - delta)
//          as bf16 128x128 tiles straight into HBM scratch, pre-swizzled in the
//          exact shared-memory layout the consumers load with one bulk copy.
//          d256: one kernel computes both (Q and dO fit in shared memory);
//          d512: one launch writes P (Q resident), a second reads P and writes
//          dS (dO resident);
//   gemm   dV = P^T dO and dK = dS^T Q (KV-major, summing every query head of
//          the GQA group in TMEM) and dQ = dS K (Q-major), each a tile-sparse
//          GEMM with a full-width (256 or 512 column) TMEM accumulator.
//
// Scratch tile layout (32 KB): [key block 0..1][query row 0..127][64 keys],
// 128-B swizzled (16-B chunk c of row r stored at chunk c ^ (r % 8)).  The
// same bytes are the K-major A operand of dQ = dS K (rows = queries) and the
// MN-major A operand of dV = P^T dO / dK = dS^T Q (rows = queries = K index).
//
// Masked pairs hold exact zeros, so consumers never re-evaluate the mask.
// This path serves the causal and sliding-window (+document) masks; vision
// metadata (whose key range per query tile is data-dependent) and workspaces
// too small for the scratch use the recompute kernels in attn_bwd.cu.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "g4_attn.cuh"
#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

constexpr int kTileBytes = 32768;  // one 128x128 bf16 scratch tile

// Scratch tiles of a band: [query head of the band][band slot], 32 KB each.
__device__ __forceinline__ int64_t band_tile_index(const MatParams& p, int head, int slot) {
  return static_cast<int64_t>(head - p.band_h0 * p.group) * p.head_cap_tiles + slot;
}
__device__ __forceinline__ uint8_t* scratch_tile(uint8_t* base, const MatParams& p, int head,
                                                 int offset, int slot) {
  return base + band_tile_index(p, head, offset + slot) * kTileBytes;
}

// The flattened query tile of band row y: the band's second range first, then
// its first, each from its last tile (the longest causal rows first), or -1.
__device__ __forceinline__ int band_qtile(const MatParams& p, int y) {
  const int n1 = p.band_g[3] - p.band_g[2];
  const int n0 = p.band_g[1] - p.band_g[0];
  if (y < n1) return p.band_g[3] - 1 - y;
  if (y < n1 + n0) return p.band_g[1] - 1 - (y - n1);
  return -1;
}
__device__ __forceinline__ int band_rows(const MatParams& p) {
  return (p.band_g[1] - p.band_g[0]) + (p.band_g[3] - p.band_g[2]);
}
__device__ __forceinline__ bool in_band(const MatParams& p, int g) {
  return (g >= p.band_g[0] && g < p.band_g[1]) || (g >= p.band_g[2] && g < p.band_g[3]);
}
// Band slots: the key tiles of the band's first range come first, those of
// the second follow.  `prefix` is a query tile's offset in the problem-wide
// prefix sum (ranges[g].z).
struct BandSlots {
  int off0, len0, off1;
  __device__ __forceinline__ BandSlots(const MatParams& p) {
    off0 = 0;
    len0 = 0;
    off1 = 0;
    if (p.band_g[1] > p.band_g[0]) {
      off0 = p.ranges[p.band_g[0]].z;
      const int4 l = p.ranges[p.band_g[1] - 1];
      len0 = l.z + l.y - off0;
    }
    if (p.band_g[3] > p.band_g[2]) off1 = p.ranges[p.band_g[2]].z;
  }
  __device__ __forceinline__ int slot(const MatParams& p, int g, int prefix) const {
    return (g >= p.band_g[0] && g < p.band_g[1]) ? prefix - off0 : len0 + prefix - off1;
  }
};

// Key tile j of query tile g (range rg): the j-th listed tile for metadata
// masks, else kt_lo + j.  List entries carry kTileEntryFull when every pair of
// the tile is allowed (the kernels then skip the mask) and kTileEntryText when
// the range rule is exact there (the kernels skip the metadata).
__device__ __forceinline__ int qtile_entry(const MatParams& p, int g, const int4& rg, int j) {
  return p.klist ? p.klist[static_cast<int64_t>(g) * p.klist_stride + j] : rg.x + j;
}
__device__ __forceinline__ int qtile_key(const MatParams& p, int g, const int4& rg, int j) {
  return qtile_entry(p, g, rg, j) & kTileEntryIndex;
}
// Position of key tile kt among query tile g's key tiles, or -1 (lists are
// sorted ascending and start at rg.x).
__device__ __forceinline__ int qtile_key_pos(const MatParams& p, int g, const int4& rg, int kt) {
  if (kt < rg.x) return -1;
  if (!p.klist) return kt < rg.x + rg.y ? kt - rg.x : -1;
  const int* l = p.klist + static_cast<int64_t>(g) * p.klist_stride;
  int lo = 0, hi = rg.y - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const int v = l[mid] & kTileEntryIndex;
    if (v == kt) return mid;
    if (v < kt) lo = mid + 1;
    else hi = mid - 1;
  }
  return -1;
}

// byte offset of the 16-B chunk holding columns [8c, 8c+8) of row r
__device__ __forceinline__ uint32_t tile_chunk_offset(int r, int c) {
  const int blk = c >> 3, ch = c & 7;
  return blk * 16384 + r * 128 + ((ch ^ (r & 7)) << 4);
}

// =====================================================================================
// plan (metadata masks): per query tile the exact list of key tiles that hold
// at least one allowed pair, each tagged kTileEntryFull when all its pairs (of
// valid rows and keys) are allowed and kTileEntryText when the range rule is
// exact on it.  One CTA per query tile, four threads per row (a quarter of the
// keys each): the row's key bound is [q - W + 1, max(q, pair_last)] (the vision
// exception has no right window cap, masks.py:55-66).  Each key tile under
// the tile's bound has its metadata staged in shared memory (the next tile's
// is loaded meanwhile); a tile without vision keys whose keys share the query
// tile's single document is classified per row in closed form, any other tile
// by testing the exact predicate on every pair.  Writes ranges[g] = (first
// listed tile, count, -, sequence); the scratch prefix follows in
// plan_qtile_ranges_kernel.  The reference builds the same incidence on the
// host (sparse_schedule.py:181-374).
// =====================================================================================
constexpr int kPlanParts = 4;
constexpr int kPlanThreads = kTileM * kPlanParts;
constexpr int kPlanKeysPerPart = kTileN / kPlanParts;

__global__ void __launch_bounds__(kPlanThreads) plan_qtile_lists_kernel(const MatParams p) {
  __shared__ __align__(16) int kvis[kTileN];
  __shared__ __align__(16) int kdoc[kTileN];
  __shared__ int lo_s, hi_s, qdoc0;
  pdl_enter();
  const int g = blockIdx.x;
  const bool packed = p.layout.packed();
  const int n = packed ? *p.n_q_tiles : p.layout.batch * p.n_qt_fixed;
  if (g >= n) return;
  int seq, qt;
  if (packed) {
    const int2 t = p.q_tiles[g];
    seq = t.x;
    qt = t.y;
  } else {
    seq = g / p.n_qt_fixed;
    qt = g % p.n_qt_fixed;
  }
  const SeqInfo si = p.layout.seq(seq);
  const int tid = threadIdx.x;
  const int r = tid & (kTileM - 1);  // query row
  const int part = tid / kTileM;     // key quarter [part * 32, + 32) of each tile
  const int W = p.mask.window;
  const int q_idx = qt * kTileM + r;
  const bool valid = q_idx < si.len_q;  // row 0 of a listed query tile always is
  const int q_abs = q_idx + si.q_off;
  int qvis = -1, qdoc = 0, lo = 0x7fffffff, hi = -1;
  if (valid) {
    if (p.mask.vis) qvis = p.mask.vis[si.meta_base + q_abs];
    if (p.mask.doc) qdoc = p.mask.doc[si.meta_base + q_abs];
    lo = W > 0 ? max(0, q_abs - W + 1) : 0;
    hi = q_abs;
    if (W > 0 && qvis >= 0)
      hi = p.mask.pair_last ? max(hi, p.mask.pair_last[si.meta_base + q_abs]) : si.len_k - 1;
    hi = min(hi, si.len_k - 1);
  }
  if (tid == 0) {
    lo_s = 0x7fffffff;
    hi_s = -1;
    qdoc0 = qdoc;
  }
  __syncthreads();
  if (part == 0 && valid && hi >= lo) {
    atomicMin(&lo_s, lo);
    atomicMax(&hi_s, hi);
  }
  const bool one_doc = __syncthreads_and(!valid || qdoc == qdoc0);
  // the range rule of this row (window bound, causal bound, end of the keys)
  const int lo_r = W > 0 ? max(0, q_abs - W + 1) : 0;
  const int hi_r = min(q_abs, si.len_k - 1);
  int* out = const_cast<int*>(p.klist) + static_cast<int64_t>(g) * p.klist_stride;
  int cnt = 0, first = 0;
  const int kt_begin = hi_s >= 0 ? lo_s / kTileN : 0;
  const int kt_end = hi_s >= 0 ? hi_s / kTileN : -1;
  // threads 0..127 stage key k0 + tid of each tile
  auto key_meta = [&](int kt, int& v, int& d) {
    const int kk = kt * kTileN + tid;
    const bool kin = tid < kTileN && kt <= kt_end && kk < si.len_k;
    v = (p.mask.vis && kin) ? p.mask.vis[si.meta_base + kk] : -1;
    d = (p.mask.doc && kin) ? p.mask.doc[si.meta_base + kk] : 0;
  };
  int nv, nd;
  key_meta(kt_begin, nv, nd);
  for (int kt = kt_begin; kt <= kt_end; ++kt) {
    const int k0 = kt * kTileN;
    const int cv = nv, cd = nd;
    key_meta(kt + 1, nv, nd);  // in flight while this tile is classified
    const bool kin = tid < kTileN && k0 + tid < si.len_k;
    __syncthreads();  // the previous tile's metadata is no longer read
    if (tid < kTileN) {
      kvis[tid] = cv;
      kdoc[tid] = cd;
    }
    const bool text = one_doc && __syncthreads_and(!kin || (cv < 0 && cd == qdoc0));
    bool any = false, all = true;
    if (valid && text) {
      if (part == 0) {
        const int k1 = min(k0 + kTileN, si.len_k) - 1;
        any = max(lo_r, k0) <= min(hi_r, k1);
        all = lo_r <= k0 && hi_r >= k0 + kTileN - 1;
      }
    } else if (valid) {
      const int kq = k0 + part * kPlanKeysPerPart;
      const int4* v4 = reinterpret_cast<const int4*>(kvis + part * kPlanKeysPerPart);
      const int4* d4 = reinterpret_cast<const int4*>(kdoc + part * kPlanKeysPerPart);
#pragma unroll
      for (int c = 0; c < kPlanKeysPerPart / 4; ++c) {
        const int4 a = v4[c], b = d4[c];
        const int av[4] = {a.x, a.y, a.z, a.w}, bd[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = kq + 4 * c + e;
          const bool ok = k < si.len_k && k >= lo && k <= hi &&
                          mask_allows(W, q_abs, k, qvis, qdoc, av[e], bd[e]);
          any |= ok;
          all &= ok;
        }
      }
    }
    const int any_t = __syncthreads_or(any);
    const int all_t = __syncthreads_and(all || !valid);
    if (any_t) {
      if (tid == 0 && cnt < p.klist_stride)
        out[cnt] = kt | (all_t ? kTileEntryFull : 0) | (text ? kTileEntryText : 0);
      if (cnt == 0) first = kt;
      ++cnt;
    }
  }
  if (tid == 0) p.ranges[g] = make_int4(first, min(cnt, p.klist_stride), 0, seq);
}

// =====================================================================================
// plan: per query tile (kt_lo, n_kt, scratch offset, sequence)
// =====================================================================================
__global__ void plan_qtile_ranges_kernel(const MatParams p) {
  __shared__ int scan[1024];
  __shared__ int carry;
  // Fixed layouts without key-tile lists compute every range from the
  // arguments alone (nothing an earlier kernel of the call writes), so they
  // wait for the predecessor only at the end: behind the backward preprocess,
  // which lets this kernel in at once, the planning runs under its loads.
  const bool packed = p.layout.packed();
  const bool late = !packed && p.klist == nullptr;
  if (!late) pdl_enter();
  const int tid = threadIdx.x;
  const int n = packed ? *p.n_q_tiles : p.layout.batch * p.n_qt_fixed;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int g = base + tid;
    int cnt = 0, kt_lo = 0, seq = 0;
    if (g < n && p.klist) {  // metadata: counts from plan_qtile_lists_kernel
      const int4 rg = p.ranges[g];
      kt_lo = rg.x;
      cnt = rg.y;
      seq = rg.w;
    } else if (g < n) {
      int qt;
      if (packed) {
        const int2 t = p.q_tiles[g];
        seq = t.x;
        qt = t.y;
      } else {
        seq = g / p.n_qt_fixed;
        qt = g % p.n_qt_fixed;
      }
      const SeqInfo si = p.layout.seq(seq);
      const int q_off = si.q_off;
      const int qa0 = qt * kTileM + q_off;
      const int qa1 = min((qt + 1) * kTileM, si.len_q) - 1 + q_off;
      const int lo = p.mask.window > 0 ? max(0, qa0 - p.mask.window + 1) : 0;
      const int hi = min(qa1, si.len_k - 1);
      if (hi >= lo) {
        kt_lo = lo / kTileN;
        cnt = hi / kTileN - kt_lo + 1;
      }
    }
    scan[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
      const int v = tid >= off ? scan[tid - off] : 0;
      __syncthreads();
      scan[tid] += v;
      __syncthreads();
    }
    if (g < n) p.ranges[g] = make_int4(kt_lo, cnt, carry + scan[tid] - cnt, seq);
    __syncthreads();
    if (tid == 1023) carry += scan[1023];
    __syncthreads();
  }
  if (late) pdl_enter();
}

// =====================================================================================
// score kernel
// =====================================================================================
enum ScoreMode : int { kScorePdS = 0, kScoreP = 1, kScoreDs = 2, kScoreFwd = 3 };

template <int D, int MODE>
struct ScoreCfg {
  static constexpr bool kS = MODE != kScoreDs;                        // S (needs Q, K)
  static constexpr bool kDP = MODE == kScorePdS || MODE == kScoreDs;   // dP (needs dO, V)
  static constexpr int kQBytes = kS ? D * kTileM * 2 : 0;
  static constexpr int kDoBytes = kDP ? D * kTileM * 2 : 0;
  static constexpr int kStages = 3;
  static constexpr int kChunksPerTile = (kS ? D / 128 : 0) + (kDP ? D / 128 : 0);
  // d512 single-product passes keep their resident operand (Q or dO) in TMEM
  // and issue TS MMAs: only B is read from shared memory, which halves the
  // shared-memory read traffic of the 128x128x512 products.  The freed shared
  // memory then holds a ring of P tiles for the dS pass.
  static constexpr bool kTS = D == 512 && MODE != kScorePdS;
  // TS variant: once the resident operand sits in TMEM its 128 KB of shared
  // memory (four 32 KB slots) extends the operand ring (more bytes in flight
  // per SM): the P pass gets 3 + 2 K stages and two slots that stage the P
  // tiles for their 32 KB bulk stores (double-buffered, so a tile's store
  // overlaps the next tile's math); the forward pass 3 + 1 K stages, the two
  // staging slots and a slot for its row-statistics exchange; the dS pass
  // 3 + 2 V stages and 2 P stages.
  static constexpr int kExtraStages = kTS ? (MODE == kScoreFwd ? 1 : 2) : (D == 256 && MODE == kScorePdS ? 2 : 0);
  static constexpr int kRingStages = kStages + kExtraStages;
  static constexpr int kPStages = 2;
  // d256 S-and-dP pass: Q and dO move into TMEM, so S = Q K^T and dP = dO V^T
  // are both TS MMAs that read only K or V from shared memory.  Q's 64 KB of
  // shared memory then hold one P and one dS staging slot, dO's 64 KB two more
  // K/V ring stages (five in all: the stream of 128 KB of K and V per key tile
  // is bound by the bytes in flight per SM).  TMEM: S at 0 and dP at 128, each
  // single-buffered (the math warps read both into registers first, then the
  // next tile's MMAs run under their arithmetic), Q at 256, dO at 384.
  static constexpr bool kQT = D == 256 && MODE == kScorePdS;
  // P tiles leave through a shared-memory staging slot and one bulk store
  // (a warp's direct 16-B row-chunk stores would touch 32 lines each).
  static constexpr bool kStageP = kTS && (MODE == kScoreP || MODE == kScoreFwd);
  // dS pass: each thread overwrites the P chunks it read from the shared P slot
  // with its dS chunks; the slot then leaves as one bulk store.
  static constexpr bool kStageDs = kTS && MODE == kScoreDs;
};

// The resident operand (Q, or dO in the dS pass) arrives in four quarters of
// its K extent, each on its own barrier, and column group g of the math warps
// moves quarter g into TMEM (TS variant): the first tile's MMAs start once
// their quarter is in place instead of after the whole 64-128 KB operand.
constexpr int kResParts = 4;

struct ScoreMisc {
  uint64_t res_full[kResParts];  // resident quarter landed (dO, when also resident, on the last)
  uint64_t a_ready[kResParts];   // resident quarter copied into TMEM (TS / QT variants)
  uint64_t ring_full[8];
  uint64_t ring_empty[8];
  uint64_t s_full[2];
  uint64_t buf_free[2];
  uint64_t p_full[4];     // P tiles in shared memory (dS pass, TS variant)
  uint64_t drain;
  uint64_t stg_free[2];   // staging slot j & 1 read by tile j's bulk store
  uint64_t stg_ready[2];  // every math thread wrote tile j's chunks (slot parity j & 1)
  uint32_t tmem_base;
  int abort;
};

// Math warps: warp w reads TMEM lanes 32*(w%4).. and the 32-column chunks
// [kChunksPerWarp*(w/4), +kChunksPerWarp) of each 128-column tile.  Sixteen
// warps (four per scheduler) hide the TMEM-load and exp latencies.
constexpr int kScoreMathWarps = 16;
constexpr int kScoreGroups = kScoreMathWarps / 4;     // column groups per row
constexpr int kChunksPerWarp = 4 / kScoreGroups;
constexpr int kScoreMathThreads = kScoreMathWarps * 32;
constexpr int kScoreThreads = kScoreMathThreads + 96;  // + producer, MMA and store warps
constexpr int kProducerWarp = kScoreMathWarps;
constexpr int kMmaWarp = kScoreMathWarps + 1;
constexpr int kStoreWarp = kScoreMathWarps + 2;

template <int D, int MODE>
__global__ void __launch_bounds__(kScoreThreads, 1)
    bwd_score_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmDO, const MatParams p) {
  using Cfg = ScoreCfg<D, MODE>;
  extern __shared__ __align__(1024) uint8_t smem[];
  pdl_enter();
  if ((smem_addr(smem) & 1023u) != 0) {
    if (p.err) atomicCAS(p.err, 0, 5);
    return;
  }
  uint8_t* q_s = smem;
  uint8_t* do_s = smem + Cfg::kQBytes;
  uint8_t* ring = do_s + Cfg::kDoBytes;
  ScoreMisc* misc = reinterpret_cast<ScoreMisc*>(ring + Cfg::kStages * 32768);

  // warp index through a shuffle: provably warp-uniform for the compiler
  const int tid = threadIdx.x, warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  // grid (heads, query tiles): the head index varies fastest in launch order, so
  // every head's longest causal rows are dispatched first (longest-first over
  // the whole grid, which keeps the tail of the launch short)
  const int head = p.band_h0 * p.group + static_cast<int>(blockIdx.x);
  const int kv_head = head / p.group;
  const bool packed = p.layout.packed();
  const int n_tiles = packed ? *p.n_q_tiles : p.layout.batch * p.n_qt_fixed;
  const int g = band_qtile(p, static_cast<int>(blockIdx.y));  // longest causal rows first
  if (g < 0 || g >= n_tiles) return;
  const int4 rg = p.ranges[g];
  const int n_kt = rg.y, seq = rg.w;
  const int t_off = BandSlots(p).slot(p, g, rg.z);
  const int qt = packed ? p.q_tiles[g].y : g % p.n_qt_fixed;
  const SeqInfo si = p.layout.seq(seq);
  const int q_off = si.q_off;
  const int64_t tok_base = packed ? si.q_base : static_cast<int64_t>(seq) * p.layout.seqlen_q;
  const bool cap_ok = t_off >= 0 && t_off + n_kt <= p.head_cap_tiles;

  if (tid == 0) {
    for (int qp = 0; qp < kResParts; ++qp) {
      mbar_init(&misc->res_full[qp], 1);
      mbar_init(&misc->a_ready[qp], kScoreMathThreads / kResParts);
    }
    for (int s = 0; s < Cfg::kRingStages; ++s) {
      mbar_init(&misc->ring_full[s], 1);
      mbar_init(&misc->ring_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&misc->s_full[b], 1);
      mbar_init(&misc->buf_free[b], kScoreMathThreads);
    }
    for (int s2 = 0; s2 < 4; ++s2) mbar_init(&misc->p_full[s2], 1);
    mbar_init(&misc->drain, 1);
    mbar_init(&misc->stg_free[0], 1);
    mbar_init(&misc->stg_free[1], 1);
    mbar_init(&misc->stg_ready[0], kScoreMathThreads);
    mbar_init(&misc->stg_ready[1], kScoreMathThreads);
    misc->abort = 0;
    fence_mbar_init();
    if (cap_ok && n_kt > 0) {
      // the resident operand is requested before TMEM allocation and the CTA
      // barrier: its 64-128 KB are the first thing every role waits for.
      // Quarter qp of the TMEM-bound operand (Q, or dO in the dS pass) lands
      // on res_full[qp]; a dO that stays in shared memory (S-and-dP pass)
      // lands on the last quarter's barrier.
      constexpr int kBpp = (D / 64) / kResParts;  // 64-element blocks per quarter
      const int qrow = si.q_base + qt * kTileM;
      const CUtensorMap* tr = Cfg::kS ? &tmQ : &tmDO;
      uint8_t* rs = Cfg::kS ? q_s : do_s;
      for (int qp = 0; qp < kResParts; ++qp) {
        const bool do_too = Cfg::kS && Cfg::kDP && qp == kResParts - 1;
        mbar_expect_tx(&misc->res_full[qp], kBpp * 16384 + (do_too ? Cfg::kDoBytes : 0));
        for (int blk = qp * kBpp; blk < (qp + 1) * kBpp; ++blk)
          tma_load_4d(rs + blk * 16384, tr, &misc->res_full[qp], blk * 64, head, qrow,
                      si.b_coord);
        if (do_too)
          for (int blk = 0; blk < D / 64; ++blk)
            tma_load_4d(do_s + blk * 16384, &tmDO, &misc->res_full[qp], blk * 64, head, qrow,
                        si.b_coord);
      }
    }
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&misc->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;
  const CtaAbort ab{&misc->abort, p.err};
  const int work = cap_ok ? n_kt : 0;
  // TMEM: PdS mode: buffer b holds S at b*256 and dP at b*256+128.  TS
  // variant: buffer b at b*128, the resident A operand (bf16 pairs) at 256.
  auto s_col = [](int b) {
    return static_cast<uint32_t>(Cfg::kTS ? b * 128 : (Cfg::kQT ? 0 : b * 256));
  };
  auto dp_col = [](int b) {
    return static_cast<uint32_t>(Cfg::kTS ? b * 128 : (Cfg::kQT ? 128 : b * 256 + 128));
  };
  uint8_t* res_area = Cfg::kS ? q_s : do_s;
  // ring stage s: the first kStages in the ring area, the rest in the
  // resident area (usable once the resident operand has moved to TMEM; the
  // d256 S-and-dP pass uses dO's area, Q's holds its staging slots)
  uint8_t* xtra_area = Cfg::kQT ? do_s : res_area;
  auto stage_ptr = [&](uint32_t st) -> uint8_t* {
    return st < static_cast<uint32_t>(Cfg::kStages) ? ring + st * 32768
                                                     : xtra_area + (st - Cfg::kStages) * 32768;
  };
  // TS dS pass: P ring after the extra V stages in the resident area; P and
  // forward passes: the staging slot there
  uint8_t* pring = res_area + Cfg::kExtraStages * 32768;
  auto stg = [&](int j) { return res_area + (Cfg::kExtraStages + (j & 1)) * 32768; };

  if (warp == kProducerWarp) {
    // whole warp: warp-uniform waits, copies issued by one elected lane
    if (work > 0) {
      uint32_t it = 0;
      bool ok = true;
      bool res_free = !(Cfg::kTS || Cfg::kQT);
      for (int j = 0; j < work && ok; ++j) {
        const int krow = si.k_base + qtile_key(p, g, rg, j) * kTileN;
        for (int c = 0; c < Cfg::kChunksPerTile && ok; ++c) {
          const uint32_t st = it % Cfg::kRingStages, ph = (it / Cfg::kRingStages) & 1;
          ++it;
          if (st >= static_cast<uint32_t>(Cfg::kStages) && !res_free) {
            for (int qp = 0; qp < kResParts && ok; ++qp)
              ok = mbar_wait(&misc->a_ready[qp], 0, ab, kDevTimeoutPeer);
            if (!ok) break;
            res_free = true;
          }
          if (!(ok = mbar_wait(&misc->ring_empty[st], ph ^ 1, ab, kDevTimeoutMma))) break;
          if (elect_one()) {
            mbar_expect_tx(&misc->ring_full[st], 32768);
            const bool is_k = Cfg::kS && c < D / 128;
            const int cc = is_k ? c : c - (Cfg::kS ? D / 128 : 0);
            for (int h = 0; h < 2; ++h)
              tma_load_4d(stage_ptr(st) + h * 16384, is_k ? &tmK : &tmV, &misc->ring_full[st],
                          (2 * cc + h) * 64, kv_head, krow, si.b_coord);
          }
          __syncwarp();
        }
      }
    }
    __syncwarp();
  } else if (warp == kStoreWarp) {
    if (lane == 0 && work > 0 && Cfg::kQT) {
      // d256 PdS: one P and one dS slot in the former Q area, refilled per tile
      bool ok = true;
      for (int j = 0; j < work && ok; ++j) {
        if (!(ok = mbar_wait(&misc->stg_ready[0], j & 1, ab, kDevTimeoutPeer))) break;
        bulk_store(scratch_tile(p.p_tiles, p, head, t_off, j), q_s, kTileBytes);
        bulk_store(scratch_tile(p.ds_tiles, p, head, t_off, j), q_s + 32768, kTileBytes);
        bulk_store_wait_read();
        mbar_arrive(&misc->stg_free[0]);
      }
      bulk_store_wait_all();
    } else if (lane == 0 && work > 0 && (Cfg::kStageP || Cfg::kStageDs)) {
      // Store warp: once every math thread has written a tile into shared
      // memory, move it to HBM with one bulk store and hand the slot back
      // (the staging slot, or the dS pass's P slot to the producer).  The math
      // warps never wait on a store, and the producer's waits never stall it.
      bool ok = true;
      auto load_p = [&](int j) {  // dS pass: P tile j into P slot j % kPStages
        const int sp = j % Cfg::kPStages;
        mbar_expect_tx(&misc->p_full[sp], kTileBytes);
        bulk_load(pring + sp * 32768, scratch_tile(p.p_tiles, p, head, t_off, j), kTileBytes,
                  &misc->p_full[sp]);
      };
      if (Cfg::kStageDs) {
        // the P slots sit in the resident area, free once dO is in TMEM
        for (int qp = 0; qp < kResParts && ok; ++qp)
          ok = mbar_wait(&misc->a_ready[qp], 0, ab, kDevTimeoutPeer);
        for (int j = 0; j < Cfg::kPStages && j < work && ok; ++j) load_p(j);
      }
      for (int j = 0; j < work && ok; ++j) {
        if (!(ok = mbar_wait(&misc->stg_ready[j & 1], (j >> 1) & 1, ab, kDevTimeoutPeer))) break;
        if (Cfg::kStageDs) {
          // the slot that held P(j) now holds dS(j): store it, then refill the
          // slot with the P tile two steps ahead (the producer never waits on
          // a P slot, so the V stream runs ahead independently)
          bulk_store(scratch_tile(p.ds_tiles, p, head, t_off, j),
                     pring + (j % Cfg::kPStages) * 32768, kTileBytes);
          bulk_store_wait_read();
          if (j + Cfg::kPStages < work) load_p(j + Cfg::kPStages);
        } else {
          bulk_store(scratch_tile(p.p_tiles, p, head, t_off, j), stg(j), kTileBytes);
          bulk_store_wait_read();
          mbar_arrive(&misc->stg_free[j & 1]);
        }
      }
      bulk_store_wait_all();  // the tiles are written before the kernel can finish
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // the whole warp runs the issue loop (warp-uniform waits, one elected lane
    // per MMA): see mbar_wait
    if (work > 0) {
      constexpr uint32_t kId = idesc_bf16(128, 128, false, false);
      const uint32_t qb = smem_addr(q_s), db = smem_addr(do_s);
      uint32_t it = 0;
      // SS variant: the whole resident area first; TS / QT: each quarter of
      // the TMEM operand before the first tile's chunks that read it
      bool ok = true;
      if (!(Cfg::kTS || Cfg::kQT))
        for (int qp = 0; qp < kResParts && ok; ++qp)
          ok = mbar_wait(&misc->res_full[qp], 0, ab, kDevTimeoutTma);
      for (int j = 0; j < work && ok; ++j) {
        const int b = j & 1;
        // S (and dP) buffers: double-buffered TMEM columns wait for tile j-2's
        // reads; the single-buffered d256 S-and-dP pair for tile j-1's
        if (!Cfg::kQT && j >= 2 &&
            !(ok = mbar_wait(&misc->buf_free[b], ((j - 2) >> 1) & 1, ab, kDevTimeoutPeer)))
          break;
        if (Cfg::kQT && j >= 1 &&
            !(ok = mbar_wait(&misc->buf_free[b ^ 1], ((j - 1) >> 1) & 1, ab, kDevTimeoutPeer)))
          break;
        tc_fence_after();
        for (int c = 0; c < Cfg::kChunksPerTile && ok; ++c) {
          const uint32_t st = it % Cfg::kRingStages, ph = (it / Cfg::kRingStages) & 1;
          ++it;
          if (!(ok = mbar_wait(&misc->ring_full[st], ph, ab, kDevTimeoutTma))) break;
          const bool is_k = Cfg::kS && c < D / 128;
          if ((Cfg::kTS || Cfg::kQT) && j == 0) {
            // K elements [128 cc, +128) of the TMEM operand: quarters
            // 2cc / kBpp .. (2cc + 1) / kBpp
            constexpr int kBpp = (D / 64) / kResParts;
            const int cq = is_k ? c : c - (Cfg::kS ? D / 128 : 0);
            for (int qp = (2 * cq) / kBpp; qp <= (2 * cq + 1) / kBpp && ok; ++qp)
              ok = mbar_wait(&misc->a_ready[qp], 0, ab, kDevTimeoutPeer);
            if (!ok) break;
          }
          tc_fence_after();
          const int cc = is_k ? c : c - (Cfg::kS ? D / 128 : 0);
          const uint32_t abase = is_k ? qb : db;
          const uint32_t dcol = is_k ? s_col(b) : dp_col(b);
          const uint32_t sb = smem_addr(stage_ptr(st));
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int gk = cc * 8 + kk;
            const uint64_t bdesc = sdesc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            if (Cfg::kTS || Cfg::kQT)  // A from TMEM: Q (or the d256 pass's dO at 384)
              umma_ts_w(tmem + dcol, tmem + ((Cfg::kQT && !is_k) ? 384 : 256) + gk * 8, bdesc,
                        kId, (cc | kk) != 0);
            else
              umma_ss_w(tmem + dcol,
                        sdesc_sw128(abase + (gk >> 2) * 16384 + (gk & 3) * 32, 16, 1024), bdesc,
                        kId, (cc | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
        }
        umma_commit_w(&misc->s_full[b]);
      }
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------- math warps: P / dS tiles to HBM ----------------
    // warp w reads TMEM lanes 32*(w%4).. (its rows) and columns [64*(w/4), +64)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int r = (warp & 3) * 32 + lane;              // row in the query tile
    const int grp = warp >> 2;                         // column group
    const int c_begin = grp * kChunksPerWarp;          // first 32-column chunk
    const int q_idx = qt * kTileM + r;
    const bool row_valid = q_idx < si.len_q;
    const int q_abs = q_idx + q_off;
    const float lse2_r =
        (row_valid && p.lse2) ? p.lse2[head * p.ws_head_stride + tok_base + q_idx] : -INFINITY;
    const float delta_r =
        (row_valid && p.delta) ? p.delta[head * p.ws_head_stride + tok_base + q_idx] : 0.f;
    const bool row_ok = row_valid && lse2_r != -INFINITY;

    const int qdoc = (row_valid && p.mask.doc) ? p.mask.doc[si.meta_base + q_abs] : 0;
    const int qvis = (row_valid && p.mask.vis) ? p.mask.vis[si.meta_base + q_abs] : -1;
    const bool meta = p.mask.has_meta();
    const int qa0 = qt * kTileM + q_off;
    const int qa1 = min((qt + 1) * kTileM, si.len_q) - 1 + q_off;
    bool ok = true;
    if ((Cfg::kTS || Cfg::kQT) && work > 0) {
      // resident Q / dO (128-B swizzled rows) -> TMEM lane r, bf16 pairs from
      // column 256; this warp copies K elements [D/4*(w/4), +D/4) of its rows
      // (quarter w/4 of the operand).
      static_assert(kScoreGroups == kResParts, "one resident quarter per column group");
      ok = mbar_wait(&misc->res_full[grp], 0, ab, kDevTimeoutTma);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        const uint8_t* src = Cfg::kS ? q_s : do_s;
        constexpr int kBlkPerGroup = (D / 64) / kScoreGroups;
#pragma unroll 1
        for (int blk = 0; blk < kBlkPerGroup; ++blk) {  // 64 K elements = 32 columns
          uint32_t v[32];
          const int dblk = grp * kBlkPerGroup + blk;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint4 w = *reinterpret_cast<const uint4*>(src + dblk * 16384 + r * 128 +
                                                            ((ch ^ (r & 7)) << 4));
            v[4 * ch + 0] = w.x;
            v[4 * ch + 1] = w.y;
            v[4 * ch + 2] = w.z;
            v[4 * ch + 3] = w.w;
          }
          tmem_st32(lane_base + 256 + dblk * 32, v);
        }
        if (Cfg::kQT) {  // dO too (it lands with the last quarter), to column 384
          if (ok && grp != kResParts - 1)
            ok = mbar_wait(&misc->res_full[kResParts - 1], 0, ab, kDevTimeoutTma);
          ok = __all_sync(0xffffffffu, ok);
#pragma unroll 1
          for (int blk = 0; blk < kBlkPerGroup && ok; ++blk) {
            uint32_t v[32];
            const int dblk = grp * kBlkPerGroup + blk;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const uint4 w = *reinterpret_cast<const uint4*>(do_s + dblk * 16384 + r * 128 +
                                                              ((ch ^ (r & 7)) << 4));
              v[4 * ch + 0] = w.x;
              v[4 * ch + 1] = w.y;
              v[4 * ch + 2] = w.z;
              v[4 * ch + 3] = w.w;
            }
            tmem_st32(lane_base + 384 + dblk * 32, v);
          }
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();  // the area is refilled by bulk copies next
      tc_fence_before();
      mbar_arrive(&misc->a_ready[grp]);
    }
    if constexpr (MODE == kScoreFwd) {
      // ---- forward pass 1: online softmax over the key tiles ----
      // Rows are shared by warps w and w+4 (64 columns each); the tile row max
      // and the final row sum are combined through shared memory, and both
      // halves take identical rescale decisions from identical inputs.
      // [2 parity][group][128] in the resident area past the extra stages (free
      // once Q is in TMEM; every math thread passed that point before use)
      float* pmax = reinterpret_cast<float*>(res_area + (Cfg::kExtraStages + 2) * 32768);
      float* lsum = pmax + 2 * kScoreGroups * 128;      // [group][128]
      const int64_t tile_base = band_tile_index(p, head, t_off);
      for (int j = tid; j < work; j += kScoreMathThreads) p.fwd_flags[tile_base + j] = 0;
      asm volatile("bar.sync 2, %0;" ::"n"(kScoreMathThreads) : "memory");
      float m_run = -INFINITY, l_half = 0.f;
      for (int j = 0; j < work; ++j) {
        const int b = j & 1;
        const int ent = qtile_entry(p, g, rg, j);
        const int k0 = (ent & kTileEntryIndex) * kTileN;
        const bool text_rule = !meta || (p.klist && (ent & kTileEntryText));
        const int cls = p.klist ? ((ent & kTileEntryFull) ? 1 : 2)
                                : (meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0, si.len_k));
        if (ok) ok = mbar_wait(&misc->s_full[b], (j >> 1) & 1, ab, kDevTimeoutMma);
        ok = __all_sync(0xffffffffu, ok);
        constexpr int kCols = 32 * kChunksPerWarp;
        float sv[kCols];
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < kChunksPerWarp; ++cc) {
            uint32_t r0[32];
            tmem_ld32(lane_base + s_col(b) + (c_begin + cc) * 32, r0);
            tmem_wait_ld();
            reg_fence32(r0);
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[cc * 32 + i] = __uint_as_float(r0[i]);
          }
          tc_fence_before();
          mbar_arrive(&misc->buf_free[b]);
        } else {
#pragma unroll
          for (int i = 0; i < kCols; ++i) sv[i] = -INFINITY;
        }
        const int kc = k0 + c_begin * 32;
        if (!(cls == 1 && kc + kCols <= si.len_k)) {
          if (text_rule) {
            // text only: the row's visible keys are one range (window bound,
            // causal bound, end of the sequence)
            const int k_lo = p.mask.window > 0 ? q_abs - p.mask.window + 1 : 0;
            const int k_hi = min(q_abs, si.len_k - 1);
#pragma unroll
            for (int i = 0; i < kCols; ++i)
              if (kc + i < k_lo || kc + i > k_hi) sv[i] = -INFINITY;
          } else {
#pragma unroll
            for (int i = 0; i < kCols; ++i) {
              const int k = kc + i;
              bool keep = k < si.len_k;
              if (cls != 1 && keep)
                keep = mask_allows(p.mask.window, q_abs, k, qvis, qdoc,
                                   p.mask.vis ? p.mask.vis[si.meta_base + k] : -1,
                                   p.mask.doc ? p.mask.doc[si.meta_base + k] : 0);
              if (!keep) sv[i] = -INFINITY;
            }
          }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int i = 0; i < kCols; ++i) mt = fmaxf(mt, sv[i]);
        float* pm = pmax + (j & 1) * kScoreGroups * 128;
        pm[grp * 128 + r] = mt * kLog2e;
        asm volatile("bar.sync 2, %0;" ::"n"(kScoreMathThreads) : "memory");
        mt = pm[r];
#pragma unroll
        for (int gi = 1; gi < kScoreGroups; ++gi) mt = fmaxf(mt, pm[gi * 128 + r]);
        float alpha = 1.f;
        if (mt > m_run + kLazyRescaleLog2) {  // lazy rescale; also the first finite tile
          // a row without any finite score so far has O = 0 and l = 0: it needs
          // no correction (alpha stays 1, the tile is not flagged for it)
          if (m_run != -INFINITY) alpha = ex2(m_run - mt);
          m_run = mt;
        }
        const float m_sub = m_run == -INFINITY ? 0.f : m_run;
        float rowsum = 0.f;
        uint8_t* ptile = scratch_tile(p.p_tiles, p, head, t_off, j);
        // staging slot j & 1 is free once tile j-2's bulk store has read it
        if (j > 1) {
          if (ok) ok = mbar_wait(&misc->stg_free[j & 1], ((j >> 1) & 1) ^ 1, ab, kDevTimeoutPeer);
          ok = __all_sync(0xffffffffu, ok);
        }
#pragma unroll
        for (int u = 0; u < kCols / 8; ++u) {
          float pe[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            pe[e] = ex2(fmaf(sv[u * 8 + e], kLog2e, -m_sub));
            rowsum += pe[e];
          }
          uint4 w;
          w.x = pack_bf16x2(pe[0], pe[1]);
          w.y = pack_bf16x2(pe[2], pe[3]);
          w.z = pack_bf16x2(pe[4], pe[5]);
          w.w = pack_bf16x2(pe[6], pe[7]);
          *reinterpret_cast<uint4*>(stg(j) + tile_chunk_offset(r, c_begin * 4 + u)) = w;
        }
        // this thread's chunks are written; the store lane moves the tile
        fence_proxy_async_smem();
        mbar_arrive(&misc->stg_ready[j & 1]);
        l_half = l_half * alpha + rowsum;
        if (grp == 0) {
          p.fwd_alpha[(tile_base + j) * 128 + r] = alpha;
          if (j > 0 && alpha != 1.f && row_valid) atomicOr(&p.fwd_flags[tile_base + j], 1);
        }
      }
      lsum[grp * 128 + r] = l_half;
      asm volatile("bar.sync 2, %0;" ::"n"(kScoreMathThreads) : "memory");
      if (grp == 0 && row_valid) {
        float l = 0.f;
#pragma unroll
        for (int gi = 0; gi < kScoreGroups; ++gi) l += lsum[gi * 128 + r];
        const float lse = l > 0.f ? (m_run + __log2f(l)) * kLn2 : -INFINITY;
        p.lse_out[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
                  static_cast<int64_t>(head) * p.lse_stride[1] + si.q_base + q_idx] = lse;
        p.fwd_inv_l[head * p.ws_head_stride + tok_base + q_idx] = l > 0.f ? 1.f / l : 0.f;
      }
    } else
    for (int j = 0; j < work; ++j) {
      const int b = j & 1;
      const int ent = qtile_entry(p, g, rg, j);
      const int k0 = (ent & kTileEntryIndex) * kTileN;
      const bool text_rule = !meta || (p.klist && (ent & kTileEntryText));
      const int cls = p.klist ? ((ent & kTileEntryFull) ? 1 : 2)
                              : (meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0, si.len_k));
      if (ok) ok = mbar_wait(&misc->s_full[b], (j >> 1) & 1, ab, kDevTimeoutMma);
      if (ok && Cfg::kTS && MODE == kScoreDs)
        ok = mbar_wait(&misc->p_full[j % Cfg::kPStages], (j / Cfg::kPStages) & 1, ab,
                       kDevTimeoutTma);
      if (Cfg::kStageP && j > 1 && ok)
        ok = mbar_wait(&misc->stg_free[j & 1], ((j >> 1) & 1) ^ 1, ab, kDevTimeoutPeer);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      const uint8_t* psm = pring + (j % Cfg::kPStages) * 32768;
      uint8_t* ptile = Cfg::kS || MODE == kScoreDs ? scratch_tile(p.p_tiles, p, head, t_off, j) : nullptr;
      uint8_t* dtile = Cfg::kDP ? scratch_tile(p.ds_tiles, p, head, t_off, j) : nullptr;
#pragma unroll 1
      for (int c = c_begin; c < c_begin + kChunksPerWarp; ++c) {
        uint32_t sr[32], dr[32];
        if (Cfg::kS && Cfg::kDP) {
          tmem_ld32(lane_base + s_col(b) + c * 32, sr);
          tmem_ld32(lane_base + dp_col(b) + c * 32, dr);
          tmem_wait_ld();
          reg_fence32(sr);
          reg_fence32(dr);
        } else if (Cfg::kS) {
          tmem_ld32(lane_base + s_col(b) + c * 32, sr);
          tmem_wait_ld();
          reg_fence32(sr);
        } else {
          tmem_ld32(lane_base + dp_col(b) + c * 32, dr);
          tmem_wait_ld();
          reg_fence32(dr);
        }
        if (c == c_begin + kChunksPerWarp - 1) {  // this warp's TMEM values are in registers
          tc_fence_before();
          mbar_arrive(&misc->buf_free[b]);
        }
        float pv[32];
        if (MODE == kScoreDs) {
          // P as written by the P-only pass (exact zeros where masked)
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 w = Cfg::kTS
                                ? *reinterpret_cast<const uint4*>(psm + tile_chunk_offset(r, c * 4 + u))
                                : *reinterpret_cast<const uint4*>(ptile + tile_chunk_offset(r, c * 4 + u));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[e]));
              pv[u * 8 + 2 * e] = f.x;
              pv[u * 8 + 2 * e + 1] = f.y;
            }
          }
        } else {
          const int kc = k0 + c * 32;
          // Fast path (warp-uniform in practice): the whole 32-key chunk is
          // inside the mask for a row with a finite LSE.
          if (cls == 1 && row_ok && kc + 32 <= si.len_k) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pv[i] = ex2(fmaf(__uint_as_float(sr[i]), kLog2e, -lse2_r));
          } else if (text_rule) {
            // text rule: the row's visible keys are one range (window bound,
            // causal bound, end of the sequence); none for a row without keys
            const int k_lo = p.mask.window > 0 ? q_abs - p.mask.window + 1 : 0;
            const int k_hi = row_ok ? min(q_abs, si.len_k - 1) : -1;
            const float sub = row_ok ? -lse2_r : 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float e = ex2(fmaf(__uint_as_float(sr[i]), kLog2e, sub));
              pv[i] = (kc + i >= k_lo && kc + i <= k_hi) ? e : 0.f;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int k = kc + i;
              bool keep = row_ok && k < si.len_k;
              if (cls != 1 && keep) {
                const int kdoc = p.mask.doc ? p.mask.doc[si.meta_base + k] : 0;
                const int kvis = p.mask.vis ? p.mask.vis[si.meta_base + k] : -1;
                keep = mask_allows(p.mask.window, q_abs, k, qvis, qdoc, kvis, kdoc);
              }
              const float e = ex2(fmaf(__uint_as_float(sr[i]), kLog2e, row_ok ? -lse2_r : 0.f));
              pv[i] = keep ? e : 0.f;
            }
          }
        }
        if (Cfg::kQT && j > 0 && c == c_begin) {
          // the staging slots are free once tile j-1's bulk stores have read them
          if (ok) ok = mbar_wait(&misc->stg_free[0], (j - 1) & 1, ab, kDevTimeoutPeer);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
        }
        if (MODE != kScoreDs) {
          uint8_t* pdst = Cfg::kQT ? q_s : (Cfg::kStageP ? stg(j) : ptile);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = pack_bf16x2(pv[u * 8 + 0], pv[u * 8 + 1]);
            w.y = pack_bf16x2(pv[u * 8 + 2], pv[u * 8 + 3]);
            w.z = pack_bf16x2(pv[u * 8 + 4], pv[u * 8 + 5]);
            w.w = pack_bf16x2(pv[u * 8 + 6], pv[u * 8 + 7]);
            *reinterpret_cast<uint4*>(pdst + tile_chunk_offset(r, c * 4 + u)) = w;
          }
        }
        if (Cfg::kDP) {
          // dS = P (dP - delta); P is exactly 0 outside the mask and dP is
          // finite for finite inputs, so no guard is needed.
          float dv[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) dv[i] = pv[i] * (__uint_as_float(dr[i]) - delta_r);
          uint8_t* ddst = Cfg::kQT ? q_s + 32768 : (Cfg::kStageDs ? const_cast<uint8_t*>(psm) : dtile);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = pack_bf16x2(dv[u * 8 + 0], dv[u * 8 + 1]);
            w.y = pack_bf16x2(dv[u * 8 + 2], dv[u * 8 + 3]);
            w.z = pack_bf16x2(dv[u * 8 + 4], dv[u * 8 + 5]);
            w.w = pack_bf16x2(dv[u * 8 + 6], dv[u * 8 + 7]);
            *reinterpret_cast<uint4*>(ddst + tile_chunk_offset(r, c * 4 + u)) = w;
          }
        }
      }
      if (Cfg::kStageP || Cfg::kStageDs || Cfg::kQT) {
        // this thread's chunks are written (dS over its P chunks in the dS
        // pass); the store lane moves the tile and frees the slot
        if (!ok) continue;
        fence_proxy_async_smem();
        mbar_arrive(&misc->stg_ready[Cfg::kQT ? 0 : j & 1]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// tile GEMM kernel: dV = P^T dO, dK = dS^T Q (KV-major) and dQ = dS K (Q-major)
// =====================================================================================
// kGemmDvDk: dV and dK in one launch.  Their KV-major CTAs have identical
// sizes (the k-steps of a key tile), so interleaving the two products doubles
// the number of CTAs of each size and evens out the end of the launch (the
// largest CTA is a smaller share of each SM's work).
enum GemmWhich : int { kGemmDv = 0, kGemmDk = 1, kGemmDq = 2, kGemmO = 3, kGemmDvDk = 4,
                       kGemmDq2 = 5 };

// dQ CTAs produce all D output columns (A loaded once); dV / dK CTAs produce
// one 256-column half each, which doubles the KV-major grid for load balance.
// PAIR (d512 dQ and forward O): the CTAs of a 2-CTA cluster take query heads
// 2i and 2i+1 of one KV group for the same query tile, so they read the same K
// (or V) rows.  Each CTA loads its own dS (or P) halves (A) and half of every
// stage's K (V) columns (B), and the leader issues cta_group::2 MMAs with
// M = 256: 48 KB per CTA and k-step instead of 80 KB, four ring stages instead
// of two.  Forward O: the MMA pauses at the union of both heads' rescale
// points; each CTA's correction warps rescale their own rows (if flagged) and
// arrive on the leader's o_ready.
template <int D, int WHICH, bool PAIR = false>
struct GemmCfg {
  // d256 dQ of the two query heads of a KV group in one CTA: both dS tiles of
  // a key tile are multiplied by one copy of its K rows (a third less operand
  // traffic than one head per CTA), into two 256-column accumulators
  static constexpr bool kDuo = WHICH == kGemmDq2;
  static constexpr bool kQMajor = WHICH == kGemmDq || WHICH == kGemmO || kDuo;  // dQ, forward O
  static constexpr int kNB = kQMajor ? D : 256;     // output columns per CTA (and head)
  static constexpr int kHalves = D / kNB;
  static constexpr int kABytes = 16384 * (kDuo ? 2 : 1);  // 128 rows x 64 deep (per head)
  static constexpr int kBBytes = 64 * (PAIR ? kNB / 2 : kNB) * 2;  // 64 deep x (this CTA's) columns
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kDuo ? 3 : (kStageBytes > 64 * 1024 ? 2 : 4);
  static_assert(!kDuo || D == 256, "two heads per CTA fill TMEM at d256");
};

constexpr int kQListCap = 2048;  // query tiles of one sequence listed in shared memory

struct GemmMisc {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t acc_full;
  uint64_t o_done;   // forward: MMAs before a rescale point completed
  uint64_t o_ready;  // forward: O rows rescaled
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  uint32_t flag_bits[64];  // forward: rescale flags of up to 2048 key tiles
  // dV / dK: the query tiles that reach this CTA's key tile, in order:
  // (query tile within the sequence, scratch slot of the key tile in its row)
  int qlist_n;             // entries, or -1 when the sequence has more query tiles than fit
  int2 qlist[kQListCap];
};

// One k-step of 64 (half a scratch tile): where A and B come from.
struct GemmStep {
  const uint8_t* a;  // scratch tile base
  int half;          // 0 / 1: which 64 of the tile's 128 contraction rows
  int b_head;        // TMA head coordinate for B
  int b_row;         // TMA token coordinate for B (first of 64 rows)
};

// Warps: 4 producer, 5 MMA, 0-3 and 6-9 epilogue.  An epilogue warp reads the
// TMEM lane quarter warp % 4 (rows 32 (warp % 4) ..), so each quarter has one
// warp in each group: warps 0-3 take the accumulator's first column half,
// warps 6-9 the second.
constexpr int kGemmThreads = 320;
constexpr int kGemmEpiThreads = 256;

template <int D, int WHICH, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    bwd_tile_gemm_kernel(const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmOut,
                         const __grid_constant__ CUtensorMap tmB2,    // kGemmDvDk: dK's B (Q)
                         const __grid_constant__ CUtensorMap tmOut2,  // kGemmDvDk: dK
                         const __grid_constant__ CUtensorMap tmA, const MatParams p) {
  using Cfg = GemmCfg<D, WHICH, PAIR>;
  static_assert(!PAIR || (Cfg::kQMajor && D == 512), "CTA pairs serve the d512 Q-major GEMMs");
  extern __shared__ __align__(1024) uint8_t smem[];
  pdl_enter();
  if ((smem_addr(smem) & 1023u) != 0) {
    if (p.err) atomicCAS(p.err, 0, 5);
    return;
  }
  GemmMisc* misc = reinterpret_cast<GemmMisc*>(smem + Cfg::kStages * Cfg::kStageBytes);
  // warp index through a shuffle: provably warp-uniform for the compiler
  const int tid = threadIdx.x, warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const bool packed = p.layout.packed();
  const int G = p.group;

  // ---- this CTA's output tile (heaviest causal work scheduled first) ----
  int seq, tile, head;  // tile: key tile (dV/dK) or query tile (dQ) within the sequence
  int qg = 0;           // dQ: global query-tile index
  int half = 0;         // dV/dK: which 256-column half
  int which = WHICH == kGemmDq2 ? kGemmDq : WHICH;  // kGemmDvDk: this CTA's product (dV or dK)
  if (Cfg::kQMajor) {
    const int n = packed ? *p.n_q_tiles : p.layout.batch * p.n_qt_fixed;
    // grid (band heads, band query tiles), head fastest: longest-first over the band
    qg = band_qtile(p, static_cast<int>(blockIdx.y));
    if (qg < 0 || qg >= n) return;
    head = p.band_h0 * G + (Cfg::kDuo ? 2 : 1) * static_cast<int>(blockIdx.x);  // (and head + 1)
    seq = p.ranges[qg].w;
    tile = packed ? p.q_tiles[qg].y : qg % p.n_qt_fixed;
  } else {
    const int per_item = p.band_nh * Cfg::kHalves;
    const int n_prod = WHICH == kGemmDvDk ? 2 : 1;  // kGemmDvDk: a dV item, then the same dK item
    const int item = p.kv_item0 + static_cast<int>(blockIdx.x) / (per_item * n_prod);
    const int r2 = blockIdx.x % (per_item * n_prod);
    if (WHICH == kGemmDvDk) which = r2 < per_item ? kGemmDv : kGemmDk;
    const int rest = r2 % per_item;
    head = p.band_h0 + rest / Cfg::kHalves;  // KV head
    half = rest % Cfg::kHalves;
    if (packed) {
      if (item >= *p.n_k_tiles) return;
      const int2 t = p.k_tiles[item];
      seq = t.x;
      tile = t.y;
    } else {
      const int nkt = (p.layout.seqlen_k + kTileN - 1) / kTileN;
      if (item >= nkt * p.layout.batch) return;
      tile = item / p.layout.batch;  // key tile 0 (most causal work) of every sequence first
      seq = item % p.layout.batch;
    }
  }
  const SeqInfo si = p.layout.seq(seq);

  // Enumerate the k-steps (two per scratch tile) in a fixed order shared by the
  // producer and the MMA thread.
  const int n_qt_seq = (si.len_q + kTileM - 1) / kTileM;
  const int first_qg = packed ? (n_qt_seq > 0 ? p.seg_first_qtile[seq] : 0) : seq * p.n_qt_fixed;
  const BandSlots bslots(p);
  // KV-major: the band's query tiles of this sequence that reach this key tile,
  // in a fixed order (first range, then second): fn(query tile in the sequence,
  // band slot of the key tile in that query tile's row); stops when fn is false.
  auto for_each_band_qtile = [&](auto&& fn) {
    for (int r = 0; r < 2; ++r) {
      const int ga = max(p.band_g[2 * r], first_qg);
      const int gb = min(p.band_g[2 * r + 1], first_qg + n_qt_seq);
      for (int gq = ga; gq < gb; ++gq) {
        const int4 rg = p.ranges[gq];
        const int pos = qtile_key_pos(p, gq, rg, tile);
        if (pos < 0) continue;
        const int t_off = bslots.slot(p, gq, rg.z);
        if (t_off < 0 || t_off + rg.y > p.head_cap_tiles) continue;  // not planned into the band
        if (!fn(gq - first_qg, t_off + pos)) return;
      }
    }
  };
  auto for_each_tile = [&](auto&& fn) {
    if (Cfg::kQMajor) {
      const int4 rg = p.ranges[qg];
      const int kv_head = head / G;
      const int t_off = bslots.slot(p, qg, rg.z);
      if (t_off < 0 || t_off + rg.y > p.head_cap_tiles) return;  // not planned into the band
      uint8_t* base = WHICH == kGemmO ? p.p_tiles : p.ds_tiles;
      for (int j = 0; j < rg.y; ++j)
        if (!fn(scratch_tile(base, p, head, t_off, j), kv_head,
                si.k_base + qtile_key(p, qg, rg, j) * kTileN))
          return;
    } else {
      uint8_t* base = which == kGemmDv ? p.p_tiles : p.ds_tiles;
      const int nl = misc->qlist_n;
      if (nl >= 0) {  // the listed query tiles
        for (int gi = 0; gi < G; ++gi) {
          const int qh = head * G + gi;
          for (int i = 0; i < nl; ++i) {
            const int2 e = misc->qlist[i];
            if (!fn(scratch_tile(base, p, qh, e.y, 0), qh, si.q_base + e.x * kTileM)) return;
          }
        }
        return;
      }
      for (int gi = 0; gi < G; ++gi) {
        const int qh = head * G + gi;
        bool go = true;
        for_each_band_qtile([&](int qt, int slot) {
          go = fn(scratch_tile(base, p, qh, slot, 0), qh, si.q_base + qt * kTileM);
          return go;
        });
        if (!go) return;
      }
    }
  };

  if (!Cfg::kQMajor && warp == 1) {
    // the query tiles that reach this key tile, gathered once by one warp
    // (32 candidates per load round): every k-step of the producer and the MMA
    // warp then reads shared memory instead of rescanning the ranges
    int cnt = 0;
    bool fits = true;
    for (int r = 0; r < 2 && fits; ++r) {
      const int ga = max(p.band_g[2 * r], first_qg);
      const int gb = min(p.band_g[2 * r + 1], first_qg + n_qt_seq);
      for (int b0 = ga; b0 < gb; b0 += 32) {
        const int gq = b0 + lane;
        bool hit = false;
        int slot = 0;
        if (gq < gb) {
          const int4 rg = p.ranges[gq];
          const int pos = qtile_key_pos(p, gq, rg, tile);
          if (pos >= 0) {
            const int t_off = bslots.slot(p, gq, rg.z);
            hit = t_off >= 0 && t_off + rg.y <= p.head_cap_tiles;
            slot = t_off + pos;
          }
        }
        const uint32_t m = __ballot_sync(0xffffffffu, hit);
        if (cnt + __popc(m) > kQListCap) {
          fits = false;
          break;
        }
        if (hit) misc->qlist[cnt + __popc(m & ((1u << lane) - 1u))] = make_int2(gq - first_qg, slot);
        cnt += __popc(m);
      }
    }
    if (lane == 0) misc->qlist_n = fits ? cnt : -1;
  }
  if (tid == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&misc->full[s], 1);
      mbar_init(&misc->empty[s], 1);
    }
    mbar_init(&misc->acc_full, 1);
    mbar_init(&misc->o_done, 1);
    // pair: one arrival per correction warp of each CTA; else one per epilogue thread
    mbar_init(&misc->o_ready, PAIR ? 2 * kGemmEpiThreads / 32 : kGemmEpiThreads);
    mbar_init(&misc->drain, 1);
    misc->abort = 0;
    fence_mbar_init();
  }
  const uint32_t crank = PAIR ? cluster_ctarank() : 0;  // 0: pair leader (or no pair)
  if (PAIR) {
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  }
  if (warp == 4) {
    if (PAIR) {
      tmem_alloc_pair(&misc->tmem_base, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&misc->tmem_base, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;
  const CtaAbort ab{&misc->abort, p.err};

  // k-step count (two per scratch tile).  Whether a query tile reaches this
  // key tile does not depend on the GQA head, so the KV-major count is the
  // length of the query-tile list times the group size.
  int n_steps = 0;
  if (Cfg::kQMajor) {
    const int4 rg = p.ranges[qg];
    const int t_off = bslots.slot(p, qg, rg.z);
    n_steps = (t_off < 0 || t_off + rg.y > p.head_cap_tiles) ? 0 : 2 * rg.y;
  } else {
    int n_qt = misc->qlist_n;
    if (n_qt < 0) {  // more query tiles than the list holds: count by scanning
      n_qt = 0;
      for_each_band_qtile([&](int, int) {
        ++n_qt;
        return true;
      });
    }
    n_steps = 2 * G * n_qt;
  }

  if (warp == 4) {
    // whole warp: warp-uniform waits, copies issued by one elected lane
    if (n_steps > 0) {
      uint32_t it = 0;
      bool ok = true;
      for_each_tile([&](const uint8_t* t, int b_head, int b_row) {
        for (int h = 0; h < 2 && ok; ++h) {
          const uint32_t st = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
          ++it;
          if (!(ok = mbar_wait(&misc->empty[st], ph ^ 1, ab, kDevTimeoutMma))) break;
          uint8_t* dst = smem + st * Cfg::kStageBytes;
          if (elect_one()) {
            if (PAIR) {
              // this CTA's dS half (one 16 KB box of the byte view of the scratch)
              // and its two 128-column slices of the 64 K rows (one per 256-wide
              // MMA); both CTAs' bytes complete on the leader's barrier
              if (crank == 0) mbar_expect_tx(&misc->full[st], 2 * Cfg::kStageBytes);
              const uint32_t lbar = mapa_shared(&misc->full[st], 0);
              const uint8_t* abase = WHICH == kGemmO ? p.p_tiles : p.ds_tiles;
              const int half_idx = static_cast<int>((t - abase) / 16384) + h;
              tma_load_3d_pair(dst, &tmA, lbar, 0, 0, half_idx);
              for (int nh = 0; nh < 2; ++nh)
                for (int bx = 0; bx < 2; ++bx)
                  tma_load_4d_pair(dst + Cfg::kABytes + (nh * 2 + bx) * 8192, &tmB, lbar,
                                   nh * 256 + static_cast<int>(crank) * 128 + bx * 64, b_head,
                                   b_row + h * 64, si.b_coord);
            } else {
              mbar_expect_tx(&misc->full[st], Cfg::kStageBytes);
              if (Cfg::kQMajor) {
                bulk_load(dst, t + h * 16384, 16384, &misc->full[st]);
                if (Cfg::kDuo)  // the next head's dS tile of the same key tile
                  bulk_load(dst + 16384, t + p.head_cap_tiles * kTileBytes + h * 16384, 16384,
                            &misc->full[st]);
              } else {
                bulk_load(dst, t + h * 8192, 8192, &misc->full[st]);
                bulk_load(dst + 8192, t + 16384 + h * 8192, 8192, &misc->full[st]);
              }
              const CUtensorMap* mb = WHICH == kGemmDvDk && which == kGemmDk ? &tmB2 : &tmB;
              for (int blk = 0; blk < Cfg::kNB / 64; ++blk)
                tma_load_4d(dst + Cfg::kABytes + blk * 8192, mb, &misc->full[st],
                            half * 256 + blk * 64, b_head, b_row + h * 64, si.b_coord);
            }
          }
          __syncwarp();
        }
        return ok;
      });
    }
    __syncwarp();
  } else if (warp == 5) {
    if (WHICH == kGemmO && n_steps > 0) {
      // gather the rescale flags into a bitmask first: a dependent global load
      // per tile on the MMA issue path would stall the tensor pipe
      const int4 rg = p.ranges[qg];
      const int t_off = bslots.slot(p, qg, rg.z);
      const int64_t flag_base = band_tile_index(p, head, t_off);
      const int64_t peer_base = band_tile_index(p, head ^ 1, t_off);
      for (int w0 = 0; w0 < (rg.y + 31) / 32 && w0 < 64; ++w0) {
        const int j = w0 * 32 + lane;
        const bool f = j < rg.y && (p.fwd_flags[flag_base + j] != 0 ||
                                    (PAIR && p.fwd_flags[peer_base + j] != 0));
        const uint32_t bits = __ballot_sync(0xffffffffu, f);
        if (lane == 0) misc->flag_bits[w0] = bits;
      }
      __syncwarp();
    }
    // the MMA issue loops run on the whole warp (warp-uniform waits, one
    // elected lane per MMA): see mbar_wait
    if (PAIR) {
      if (n_steps > 0 && crank == 0) {
        // leader: M = 256 (both CTAs' query rows), N = 256 per MMA (128
        // columns from each CTA's stage)
        constexpr uint32_t kId = idesc_bf16(256, 256, false, true);
        const uint32_t sb0 = smem_addr(smem);
        bool ok = true;
        int events = 0;
        for (int it = 0; it < n_steps && ok; ++it) {
          const int tj = it >> 1;  // scratch tile of this half-step
          if (WHICH == kGemmO && (it & 1) == 0 && tj > 0 &&
              ((misc->flag_bits[(tj >> 5) & 63] >> (tj & 31)) & 1u)) {
            // both CTAs' correction warps rescale O once every earlier product completed
            umma_commit_pair_both_w(&misc->o_done);
            if (!(ok = mbar_wait_cluster(&misc->o_ready, events & 1, ab, kDevTimeoutPeer)))
              break;
            tc_fence_after();
            ++events;
          }
          const uint32_t st = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
          if (!(ok = mbar_wait(&misc->full[st], ph, ab, kDevTimeoutTma))) break;
          tc_fence_after();
          const uint32_t a = sb0 + st * Cfg::kStageBytes;
          const uint32_t bb = a + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adesc = sdesc_sw128(a + kk * 32, 16, 1024);
#pragma unroll
            for (int nh = 0; nh < 2; ++nh)
              umma_ss_pair_w(tmem + nh * 256, adesc,
                             sdesc_sw128(bb + nh * 16384 + kk * 2048, 8192, 1024), kId,
                             !(it == 0 && kk == 0));
          }
          umma_commit_pair_both_w(&misc->empty[st]);
        }
        umma_commit_pair_both_w(&misc->acc_full);
        umma_commit_pair_both_w(&misc->drain);
        mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
      }
    } else if (n_steps > 0) {
      constexpr uint32_t kId = idesc_bf16(128, 256, !Cfg::kQMajor, true);
      const uint32_t sb0 = smem_addr(smem);
      uint32_t it = 0;
      bool ok = true;
      int tile_j = 0, events = 0;
      for_each_tile([&](const uint8_t*, int, int) {
        // forward: before the first product of a flagged tile, let the
        // correction warps rescale O once every earlier product completed
        if (WHICH == kGemmO && tile_j > 0 &&
            ((misc->flag_bits[(tile_j >> 5) & 63] >> (tile_j & 31)) & 1u)) {
          umma_commit_w(&misc->o_done);
          if (!(ok = mbar_wait(&misc->o_ready, events & 1, ab, kDevTimeoutPeer)))
            return false;
          tc_fence_after();
          ++events;
        }
        ++tile_j;
        for (int h = 0; h < 2 && ok; ++h) {
          const uint32_t st = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
          const uint32_t first = it == 0;
          ++it;
          if (!(ok = mbar_wait(&misc->full[st], ph, ab, kDevTimeoutTma))) break;
          tc_fence_after();
          const uint32_t a = sb0 + st * Cfg::kStageBytes;
          const uint32_t bb = a + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adesc = Cfg::kQMajor ? sdesc_sw128(a + kk * 32, 16, 1024)
                                                : sdesc_sw128(a + kk * 2048, 8192, 1024);
#pragma unroll
            for (int nh = 0; nh < Cfg::kNB / 256; ++nh)
              umma_ss_w(tmem + nh * 256, adesc,
                        sdesc_sw128(bb + nh * 32768 + kk * 2048, 8192, 1024), kId,
                        !(first && kk == 0));
            if (Cfg::kDuo)  // second head: its dS half against the same K rows
              umma_ss_w(tmem + 256, sdesc_sw128(a + 16384 + kk * 32, 16, 1024),
                        sdesc_sw128(bb + kk * 2048, 8192, 1024), kId, !(first && kk == 0));
          }
          umma_commit_w(&misc->empty[st]);
        }
        return ok;
      });
      umma_commit_w(&misc->acc_full);
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: TMEM -> bf16 rows ----------------
    // row er of the tile (TMEM lane quarter warp % 4); columns [c_lo, c_hi)
    // in 32-column chunks: the first or second half of the accumulator
    bool ok = true;
    const int er = (warp & 3) * 32 + lane;
    const int ehalf = warp < 4 ? 0 : 1;
    const uint32_t lane_base0 = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    if (WHICH == kGemmO && n_steps > 0) {
      // correction: apply the forward's lazy rescale factors at flagged tiles
      const int4 rg = p.ranges[qg];
      const int t_off = bslots.slot(p, qg, rg.z);
      const int64_t tile_base = band_tile_index(p, head, t_off);
      const int64_t peer_base = band_tile_index(p, head ^ 1, t_off);
      int events = 0;
      for (int j = 1; j < rg.y && ok; ++j) {
        if (!p.fwd_flags[tile_base + j] && !(PAIR && p.fwd_flags[peer_base + j])) continue;
        ok = mbar_wait(&misc->o_done, events & 1, ab, kDevTimeoutMma);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float a = p.fwd_alpha[(tile_base + j) * 128 + er];
        if (__any_sync(0xffffffffu, a != 1.f)) {
#pragma unroll 1
          for (int c = ehalf * (D / 64); c < (ehalf + 1) * (D / 64); c += 2) {
            uint32_t r0[32], r1[32];
            tmem_ld32(lane_base0 + c * 32, r0);
            tmem_ld32(lane_base0 + c * 32 + 32, r1);
            tmem_wait_ld();
            reg_fence32(r0);
            reg_fence32(r1);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              r0[i] = __float_as_uint(__uint_as_float(r0[i]) * a);
              r1[i] = __float_as_uint(__uint_as_float(r1[i]) * a);
            }
            tmem_st32(lane_base0 + c * 32, r0);
            tmem_st32(lane_base0 + c * 32 + 32, r1);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        if (PAIR) {  // one arrival per warp on the leader's barrier
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(&misc->o_ready, 0));
        } else {
          mbar_arrive(&misc->o_ready);
        }
        ++events;
      }
    }
    if (ok && n_steps > 0) ok = mbar_wait(&misc->acc_full, 0, ab, kDevTimeoutMma);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool have = ok && n_steps > 0;
    const uint32_t lane_base = lane_base0;  // the first (or only) accumulator
    const int row = tile * 128 + er;
    constexpr int kHalfChunks = Cfg::kNB / 64;  // 32-column chunks per epilogue warp
    const int c_lo = ehalf * kHalfChunks;
    const bool row_valid = Cfg::kQMajor ? row < si.len_q : row < si.len_k;
    const bool acc = Cfg::kQMajor ? (WHICH == kGemmDq && p.acc_q != 0) : p.acc_kv != 0;
    if (acc) {
      // fp32 accumulation: this CTA's product is added into an fp32 tensor (a
      // band's partial dV / dK, or a caller's gradient accumulator).  A CTA
      // without k-steps adds nothing: no query tile of the band reaches it.
      if (n_steps > 0) {
        const int len_a = Cfg::kQMajor ? si.len_q : si.len_k;
        // uniform over the column half, as for the bf16 stores below
        const bool via_red =
            bar_red_and(2 + ehalf, kGemmEpiThreads / 2, have && tile * 128 + 128 <= len_a);
        if (via_red) {
          const int tok0 = (Cfg::kQMajor ? si.q_base : si.k_base) + tile * 128;
          const CUtensorMap* mo = WHICH == kGemmDvDk && which == kGemmDk ? &tmOut2 : &tmOut;
          const bool issuer = lane == 0 && (warp & 3) == 0;
          // 32 fp32 columns (128 B per row, 16 KB per chunk) staged at a time,
          // four chunks per half in flight before the staging area is reused
          constexpr int kRound = 4;
          uint8_t* stg_half = smem + ehalf * kRound * 16384;
#pragma unroll 1
          for (int c0 = 0; c0 < kHalfChunks; c0 += kRound) {
            if (c0 > 0) {  // the previous round's reduces have read the staging area
              if (issuer) bulk_store_wait_read();
              asm volatile("bar.sync %0, %1;" ::"r"(2 + ehalf), "n"(kGemmEpiThreads / 2) : "memory");
            }
#pragma unroll 1
            for (int cc = 0; cc < kRound && c0 + cc < kHalfChunks; ++cc) {
              const int c = c_lo + c0 + cc;
              uint32_t r[32];
              tmem_ld32(lane_base + c * 32, r);
              tmem_wait_ld();
              reg_fence32(r);
              uint8_t* rowp = stg_half + cc * 16384 + er * 128;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                *reinterpret_cast<uint4*>(rowp + ((i ^ (er & 7)) << 4)) =
                    make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
              fence_proxy_async_smem();
              asm volatile("bar.sync %0, %1;" ::"r"(2 + ehalf), "n"(kGemmEpiThreads / 2) : "memory");
              if (issuer) {
                tma_reduce_add_4d(mo, stg_half + cc * 16384, half * 256 + c * 32, head, tok0,
                                  si.b_coord);
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
              }
            }
          }
          if (issuer) bulk_store_wait_read();
        } else if (have) {
          // a partial tile of a packed segment: element atomics on valid rows
          float* adst;
          if (which == kGemmDq)
            adst = p.dq_acc + static_cast<int64_t>(si.b_coord) * p.dq_acc_stride[0] +
                   static_cast<int64_t>(si.q_base + row) * p.dq_acc_stride[1] +
                   static_cast<int64_t>(head) * p.dq_acc_stride[2];
          else if (which == kGemmDv)
            adst = p.dv_acc + static_cast<int64_t>(si.b_coord) * p.dv_acc_stride[0] +
                   static_cast<int64_t>(si.k_base + row) * p.dv_acc_stride[1] +
                   static_cast<int64_t>(head) * p.dv_acc_stride[2];
          else
            adst = p.dk_acc + static_cast<int64_t>(si.b_coord) * p.dk_acc_stride[0] +
                   static_cast<int64_t>(si.k_base + row) * p.dk_acc_stride[1] +
                   static_cast<int64_t>(head) * p.dk_acc_stride[2];
          adst += half * 256;
#pragma unroll 1
          for (int c = c_lo; c < c_lo + kHalfChunks; ++c) {
            uint32_t r[32];
            tmem_ld32(lane_base + c * 32, r);
            tmem_wait_ld();
            reg_fence32(r);
            if (row_valid)
#pragma unroll
              for (int i = 0; i < 32; ++i) atomicAdd(adst + c * 32 + i, __uint_as_float(r[i]));
          }
        }
      }
    } else {
    for (int u = 0; u < (Cfg::kDuo ? 2 : 1); ++u) {  // kDuo: both heads' accumulators
    const int hu = head + u;
    const uint32_t lane_base = lane_base0 + u * 256;
    uint8_t* const stg_out = smem + u * 65536;
    float out_scale = 1.f;
    __nv_bfloat16* dst;
    if (WHICH == kGemmO) {
      const int64_t tok = (packed ? si.q_base : static_cast<int64_t>(seq) * p.layout.seqlen_q) + row;
      out_scale = row_valid ? p.fwd_inv_l[head * p.ws_head_stride + tok] : 0.f;
      dst = p.o + static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
            static_cast<int64_t>(si.q_base + row) * p.o_stride[1] + static_cast<int64_t>(head) * p.o_stride[2];
    } else if (which == kGemmDq)
      dst = p.dq + static_cast<int64_t>(si.b_coord) * p.dq_stride[0] +
            static_cast<int64_t>(si.q_base + row) * p.dq_stride[1] + static_cast<int64_t>(hu) * p.dq_stride[2];
    else if (which == kGemmDv)
      dst = p.dv + static_cast<int64_t>(si.b_coord) * p.dv_stride[0] +
            static_cast<int64_t>(si.k_base + row) * p.dv_stride[1] + static_cast<int64_t>(head) * p.dv_stride[2];
    else
      dst = p.dk + static_cast<int64_t>(si.b_coord) * p.dk_stride[0] +
            static_cast<int64_t>(si.k_base + row) * p.dk_stride[1] + static_cast<int64_t>(head) * p.dk_stride[2];
    dst += half * 256;
    // A full 128-row tile leaves through shared memory: each thread writes its
    // row in the 128-B swizzled layout into the operand ring (idle once every
    // MMA has completed) and one thread issues a TMA store per 64-column block,
    // instead of 16-B row-chunk stores that touch 32 lines per warp store.  A
    // partial tile of a packed segment would spill into the next segment, so
    // partial tiles keep the direct stores.
    const int seq_len = Cfg::kQMajor ? si.len_q : si.len_k;
    // The choice must be the same for all 128 threads of a column half: the
    // TMA branch meets named barrier 2 + ehalf once per block, the direct
    // branch never.  `have` is only warp-uniform (one warp's bounded wait may
    // expire while another's passes), so the half takes the TMA branch only
    // when every one of its threads has the accumulator (an AND-reduction on
    // the same named barrier, which every epilogue thread reaches).
    const bool via_tma =
        bar_red_and(2 + ehalf, kGemmEpiThreads / 2, have && tile * 128 + 128 <= seq_len);
    if (via_tma) {
      // two 32-column chunks per TMEM wait (one 64-column block of the
      // 128-B swizzled staging layout); each group of four warps syncs on its
      // own named barrier once a block holds all 128 rows, and its first warp
      // stores that block at once, so the stores overlap the later blocks
      const int tok0 = (Cfg::kQMajor ? si.q_base : si.k_base) + tile * 128;
      const CUtensorMap* mo = WHICH == kGemmDvDk && which == kGemmDk ? &tmOut2 : &tmOut;
      const bool issuer = lane == 0 && (warp & 3) == 0;  // warp 0 (first half), warp 8 (second)
#pragma unroll 1
      for (int c = c_lo; c < c_lo + kHalfChunks; c += 2) {
        uint32_t r[2][32];
        tmem_ld32(lane_base + c * 32, r[0]);
        tmem_ld32(lane_base + c * 32 + 32, r[1]);
        tmem_wait_ld();
        reg_fence32(r[0]);
        reg_fence32(r[1]);
        uint8_t* rowp = stg_out + (c >> 1) * 16384 + er * 128;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4*>(rowp + (((hh * 4 + i) ^ (er & 7)) << 4)) =
                make_uint4(pack_bf16x2(__uint_as_float(r[hh][8 * i + 0]) * out_scale,
                                       __uint_as_float(r[hh][8 * i + 1]) * out_scale),
                           pack_bf16x2(__uint_as_float(r[hh][8 * i + 2]) * out_scale,
                                       __uint_as_float(r[hh][8 * i + 3]) * out_scale),
                           pack_bf16x2(__uint_as_float(r[hh][8 * i + 4]) * out_scale,
                                       __uint_as_float(r[hh][8 * i + 5]) * out_scale),
                           pack_bf16x2(__uint_as_float(r[hh][8 * i + 6]) * out_scale,
                                       __uint_as_float(r[hh][8 * i + 7]) * out_scale));
        fence_proxy_async_smem();
        asm volatile("bar.sync %0, %1;" ::"r"(2 + ehalf), "n"(kGemmEpiThreads / 2) : "memory");
        if (issuer) {
          tma_store_4d(mo, stg_out + (c >> 1) * 16384, half * 256 + (c >> 1) * 64, hu, tok0,
                       si.b_coord);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      // the staging area is read before the CTA's shared memory is released;
      // the global writes complete with the grid
      if (issuer) bulk_store_wait_read();
    } else {
#pragma unroll 1
      for (int c = c_lo; c < c_lo + kHalfChunks; ++c) {
        uint32_t r[32];
        if (have) {
          tmem_ld32(lane_base + c * 32, r);
          tmem_wait_ld();
          reg_fence32(r);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        if (row_valid) {
          uint4* out = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            out[i] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * i + 0]) * out_scale,
                                            __uint_as_float(r[8 * i + 1]) * out_scale),
                                pack_bf16x2(__uint_as_float(r[8 * i + 2]) * out_scale,
                                            __uint_as_float(r[8 * i + 3]) * out_scale),
                                pack_bf16x2(__uint_as_float(r[8 * i + 4]) * out_scale,
                                            __uint_as_float(r[8 * i + 5]) * out_scale),
                                pack_bf16x2(__uint_as_float(r[8 * i + 6]) * out_scale,
                                            __uint_as_float(r[8 * i + 7]) * out_scale));
        }
      }
    }
    }  // heads
    }  // bf16 outputs
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the peer's MMAs into this CTA's TMEM are complete
  if (warp == 4) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, 512);
    else
      tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// fp32 -> bf16 rows: the final dV / dK of a multi-band backward
// =====================================================================================
// src: [row][head][d] fp32, contiguous (row = batch * rows_per_batch + token);
// dst: bf16 with element strides (batch, token, head).  Eight values per step.
__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, int64_t rows, int heads, int d,
                                     __nv_bfloat16* dst, int64_t s0, int64_t s1, int64_t s2,
                                     int64_t rows_per_batch) {
  pdl_enter();
  const int64_t n8 = rows * heads * (d / 8);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int c = static_cast<int>(e % d);
    const int64_t rh = e / d;
    const int h = static_cast<int>(rh % heads);
    const int64_t row = rh / heads;
    const int64_t b = row / rows_per_batch, t = row % rows_per_batch;
    const float4 x0 = reinterpret_cast<const float4*>(src + e)[0];
    const float4 x1 = reinterpret_cast<const float4*>(src + e)[1];
    *reinterpret_cast<uint4*>(dst + b * s0 + t * s1 + h * s2 + c) =
        make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                   pack_bf16x2(x1.z, x1.w));
  }
}

// =====================================================================================
// launchers
// =====================================================================================
int launch_cast_f32_bf16(const float* src, int64_t rows, int heads, int d, __nv_bfloat16* dst,
                         const int64_t* dst_stride, int batch, int64_t rows_per_batch,
                         cudaStream_t stream) {
  (void)batch;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n8 = rows * heads * (d / 8);
  const int64_t blocks = std::min<int64_t>((n8 + 255) / 256, int64_t(sms) * 8);
  if (blocks <= 0) return 0;
  cudaError_t e = launch_chained(cast_f32_bf16_kernel, dim3(static_cast<unsigned>(blocks)),
                                 dim3(256), 0, stream, src, rows, heads, d, dst, dst_stride[0],
                                 dst_stride[1], dst_stride[2], rows_per_batch);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

int launch_plan_qtile_lists(const MatParams& p, int n_qt_total, cudaStream_t stream) {
  if (n_qt_total <= 0) return 0;
  cudaError_t e = launch_chained(plan_qtile_lists_kernel, dim3(n_qt_total), dim3(kPlanThreads), 0,
                                 stream, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

int launch_plan_qtile_ranges(const MatParams& p, cudaStream_t stream) {
  cudaError_t e = launch_chained(plan_qtile_ranges_kernel, dim3(1), dim3(1024), 0, stream, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

template <int D, int MODE>
static int launch_score_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const CUtensorMap& tdo, const MatParams& p, int grid_x,
                             cudaStream_t stream) {
  using Cfg = ScoreCfg<D, MODE>;
  const int smem = Cfg::kQBytes + Cfg::kDoBytes + Cfg::kStages * 32768 + sizeof(ScoreMisc);
  cudaError_t e = cudaFuncSetAttribute(bwd_score_kernel<D, MODE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = launch_chained(bwd_score_kernel<D, MODE>, dim3(p.band_nh * p.group, grid_x),
                     dim3(kScoreThreads), smem, stream, tq, tk, tv, tdo, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

int launch_bwd_score(int d, int pass, const CUtensorMap& tq, const CUtensorMap& tk,
                     const CUtensorMap& tv, const CUtensorMap& tdo, const MatParams& p, int grid_x,
                     cudaStream_t stream) {
  if (pass == 2) return launch_score_impl<512, kScoreFwd>(tq, tk, tv, tdo, p, grid_x, stream);
  if (d == 256) return launch_score_impl<256, kScorePdS>(tq, tk, tv, tdo, p, grid_x, stream);
  if (pass == 0) return launch_score_impl<512, kScoreP>(tq, tk, tv, tdo, p, grid_x, stream);
  return launch_score_impl<512, kScoreDs>(tq, tk, tv, tdo, p, grid_x, stream);
}

template <int D, int WHICH, bool PAIR = false>
static int launch_gemm_impl(const CUtensorMap& tb, const CUtensorMap& tout, const CUtensorMap& ta,
                            const CUtensorMap& tb2, const CUtensorMap& tout2, const MatParams& p,
                            int grid_x, int grid_y, cudaStream_t stream) {
  using Cfg = GemmCfg<D, WHICH, PAIR>;
  if (!Cfg::kQMajor) {  // KV-major: (key tile, [product,] KV head, half) all along x
    grid_x *= grid_y * Cfg::kHalves * (WHICH == kGemmDvDk ? 2 : 1);
    grid_y = 1;
  }
  if (Cfg::kDuo) grid_y /= 2;  // head pairs
  const int smem = Cfg::kStages * Cfg::kStageBytes + sizeof(GemmMisc);
  auto kernel = bwd_tile_gemm_kernel<D, WHICH, PAIR>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = Cfg::kQMajor ? dim3(grid_y, grid_x) : dim3(grid_x, grid_y);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // chained: pdl_enter
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (PAIR) {  // query heads 2i, 2i+1 (grid x) form a cluster
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  e = cudaLaunchKernelEx(&cfg, kernel, tb, tout, tb2, tout2, ta, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

bool gemm_pairs_ok(int d, int which, const MatParams& p) {
  return d == 512 && (which == kGemmDq || which == kGemmO) && (p.group % 2) == 0 &&
         (p.num_q_heads % 2) == 0;
}

int launch_bwd_tile_gemm(int d, int which, const CUtensorMap& tb, const CUtensorMap& tout,
                         const CUtensorMap* ta, const MatParams& p, int grid_x, int grid_y,
                         cudaStream_t stream) {
  const CUtensorMap& a = ta ? *ta : tb;  // only read by the pair variant
  if (d == 256) {
    if (which == kGemmDv)
      return launch_gemm_impl<256, kGemmDv>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
    if (which == kGemmDk)
      return launch_gemm_impl<256, kGemmDk>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
    if (p.group % 2 == 0 && p.acc_q == 0 && grid_y % 2 == 0)  // head pairs of a KV group
      return launch_gemm_impl<256, kGemmDq2>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
    return launch_gemm_impl<256, kGemmDq>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
  }
  if (which == kGemmDv)
    return launch_gemm_impl<512, kGemmDv>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
  if (which == kGemmDk)
    return launch_gemm_impl<512, kGemmDk>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
  if (which == kGemmO) {
    if (ta && gemm_pairs_ok(d, which, p))
      return launch_gemm_impl<512, kGemmO, true>(tb, tout, *ta, tb, tout, p, grid_x, grid_y,
                                                 stream);
    return launch_gemm_impl<512, kGemmO>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
  }
  if (ta && gemm_pairs_ok(d, which, p))
    return launch_gemm_impl<512, kGemmDq, true>(tb, tout, *ta, tb, tout, p, grid_x, grid_y,
                                                stream);
  return launch_gemm_impl<512, kGemmDq>(tb, tout, a, tb, tout, p, grid_x, grid_y, stream);
}

int launch_bwd_tile_gemm_dvdk(int d, const CUtensorMap& tdo, const CUtensorMap& tdv,
                              const CUtensorMap& tq, const CUtensorMap& tdk, const MatParams& p,
                              int grid_x, int grid_y, cudaStream_t stream) {
  if (d == 256)
    return launch_gemm_impl<256, kGemmDvDk>(tdo, tdv, tdo, tq, tdk, p, grid_x, grid_y, stream);
  return launch_gemm_impl<512, kGemmDvDk>(tdo, tdv, tdo, tq, tdk, p, grid_x, grid_y, stream);
}

}  // namespace g4
