// Gemma-4 attention backward for sm_100a (TMA + tcgen05, accumulators in TMEM).
//
// Three launches on the caller's stream:
//   1. preprocess : delta = rowsum(dO * O) - dLSE and lse2 = LSE * log2(e) per
//                   (head, token) into the workspace (one warp per row);
//   2. dQ kernel  : Q-major.  CTA = (128-query tile, query head, 256-wide dQ
//                   slab).  Per 128-key tile: S = Q K^T and dP = dO V^T into
//                   TMEM, the four softmax warps turn them into
//                   dS = P * (dP - delta) (bf16, written back over S), then
//                   dQ += dS K with dS read from TMEM;
//   3. dK/dV kernel: KV-major.  CTA = (128-key tile, KV head, 128-wide dK/dV
//                   slab).  Loops over every query head of the GQA group and
//                   every query tile the mask lets reach the key tile:
//                   S^T = K Q^T, dP^T = V dO^T, P^T and dS^T (bf16, written
//                   back over S^T / dP^T), then dV += P^T dO and dK += dS^T Q.
//                   The GQA reduction happens in TMEM, so dK/dV need no atomics
//                   and are deterministic.
// The softmax scale is 1.0, so no scale factors appear.  Keys outside every
// query's mask receive exact zeros.  Fully masked query rows (LSE = -inf)
// contribute nothing.
//
// Reference interfaces replaced: FA4's autograd backward for the local
// adapters (src/gemma4_fa4/h100.py:766-910) and
// flash_attn.cute.interface._flash_attn_bwd_gemma4_global_d512
// (patches/flash-attention/0002-sm90-gemma4-d512-forward-backward.patch:1021-1512),
// whose split preprocess / dKV / dQ / postprocess launches and fp32 global
// workspaces this design does not need.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/gemma4_b200.h"
#include "g4_attn.cuh"
#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

// =====================================================================================
// 1. preprocess
// =====================================================================================
// One warp per 512 features of (token, head) rows: a row of d512, two rows of
// d256.  Every load of the warp is issued before the first multiply (two
// 16-B loads of O and dO per lane and row of 256 features), so that a warp
// keeps 2 KB in flight whatever the head dimension.
template <int DV>
struct PreCfg {
  static constexpr int kRows = DV == 256 ? 2 : 1;  // rows per warp
  static constexpr int kIters = DV / 256;           // 16-B loads per lane and row
};

template <int DV>
__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const BwdParams p, int64_t tokens_q,
                                                             int early_trigger) {
  constexpr int kRows = PreCfg<DV>::kRows, kIters = PreCfg<DV>::kIters;
  // A successor that waits for this kernel only at its own end (the one-CTA
  // range planner of fixed layouts) is let in at once: it plans under the loads.
  if (early_trigger) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // This kernel reads only the call's inputs (O, dO, LSE, dLSE: written before
  // the call's plain-launched workspace reset started) and writes delta and
  // log2 LSE, which no kernel of the call before it touches, so it waits for its
  // predecessor (pdl_enter) only at its end: the reset and the packed-layout
  // planning run under its loads, and its completion still implies theirs.
  const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = tokens_q * p.num_q_heads;
  const int64_t row0 = warp_id * kRows;
  if (row0 >= rows) {
    pdl_enter();
    return;
  }
  uint4 ov[kRows][kIters], gv[kRows][kIters];
  int64_t bs[kRows], ss[kRows], tk[kRows];
  int hs[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int64_t row = min(row0 + r, rows - 1);  // a missing last row repeats (unwritten)
    hs[r] = static_cast<int>(row % p.num_q_heads);
    tk[r] = row / p.num_q_heads;
    if (p.layout.packed()) {
      bs[r] = 0;
      ss[r] = tk[r];
    } else {
      bs[r] = tk[r] / p.layout.seqlen_q;
      ss[r] = tk[r] % p.layout.seqlen_q;
    }
    const __nv_bfloat16* o =
        p.o + bs[r] * p.o_stride[0] + ss[r] * p.o_stride[1] + hs[r] * p.o_stride[2];
    const __nv_bfloat16* g =
        p.dout + bs[r] * p.do_stride[0] + ss[r] * p.do_stride[1] + hs[r] * p.do_stride[2];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      ov[r][it] = *reinterpret_cast<const uint4*>(o + it * 256 + lane * 8);
      gv[r][it] = *reinterpret_cast<const uint4*>(g + it * 256 + lane * 8);
    }
  }
  float acc[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    acc[r] = 0.f;
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov[r][it]);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[r][it]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __bfloat1622float2(o2[i]);
        const float2 d = __bfloat1622float2(g2[i]);
        acc[r] = fmaf(a.x, d.x, acc[r]);
        acc[r] = fmaf(a.y, d.y, acc[r]);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
  if (lane < kRows && row0 + lane < rows) {
    // lane r writes row r (the values are selected without dynamic indexing)
    float a = acc[0];
    int64_t b = bs[0], s = ss[0], tok = tk[0];
    int h = hs[0];
#pragma unroll
    for (int r = 1; r < kRows; ++r)
      if (lane == r) {
        a = acc[r];
        b = bs[r];
        s = ss[r];
        tok = tk[r];
        h = hs[r];
      }
    const int64_t li = b * p.lse_stride[0] + h * p.lse_stride[1] + s;
    const float lse = p.lse[li];
    const float dl = p.dlse ? p.dlse[li] : 0.f;
    const int64_t wi = h * p.ws_head_stride + tok;
    p.delta[wi] = a - (isfinite(dl) ? dl : 0.f);
    p.lse2[wi] = lse == -INFINITY ? -INFINITY : lse * kLog2e;
  }
  pdl_enter();
}

int launch_bwd_preprocess(const BwdParams& p, int head_dim_v, int64_t tokens_q,
                          bool early_trigger, cudaStream_t stream) {
  const int64_t rows = tokens_q * p.num_q_heads;
  const int threads = 256;
  const int per_warp = head_dim_v == 256 ? PreCfg<256>::kRows : PreCfg<512>::kRows;
  const int64_t warps = (rows + per_warp - 1) / per_warp;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (blocks == 0) return 0;
  const dim3 grid(static_cast<unsigned>(blocks));
  const cudaError_t e =
      head_dim_v == 256
          ? launch_chained(bwd_preprocess_kernel<256>, grid, dim3(threads), 0, stream, p, tokens_q,
                           early_trigger ? 1 : 0)
          : launch_chained(bwd_preprocess_kernel<512>, grid, dim3(threads), 0, stream, p, tokens_q,
                           early_trigger ? 1 : 0);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

// Shared pieces of the two main kernels ---------------------------------------------
struct BwdMisc {
  uint64_t res_full;       // resident operands landed
  uint64_t ring_full[4];
  uint64_t ring_empty[4];
  uint64_t s_full;         // S and dP (or S^T and dP^T) computed
  uint64_t ds_full;        // softmax warps wrote dS (and P^T)
  uint64_t step_done;      // accumulation MMAs of a step completed
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int lo;
  int hi;
  int pad[4];
  float col_lse2[kTileN];
  float col_delta[kTileN];
  int col_vis[kTileN];
  int col_doc[kTileN];
};

constexpr int kStageBytes = 32768;
constexpr int kBwdStages = 3;
constexpr int kBwdMiscBytes = (sizeof(BwdMisc) + 15) / 16 * 16;
enum : int { kDevBadSmemAlign = 5 };

// The operand tiles need 1024-B alignment for the 128-B swizzle; the dynamic
// shared window starts 1024-B aligned when a kernel has no static shared
// memory.  No slack is reserved (the tiles fill all 227 KB), so this is
// verified instead of assumed: a misaligned base records an error and the CTA
// returns before touching shared memory.
__device__ __forceinline__ bool smem_base_ok(const void* base, int* err) {
  if ((smem_addr(base) & 1023u) == 0) return true;
  if (err) atomicCAS(err, 0, kDevBadSmemAlign);
  return false;
}

__device__ __forceinline__ void ld_chunk_pair(uint32_t a_addr, uint32_t b_addr, uint32_t (&a)[32],
                                              uint32_t (&b)[32]) {
  tmem_ld32(a_addr, a);
  tmem_ld32(b_addr, b);
  tmem_wait_ld();
  reg_fence32(a);
  reg_fence32(b);
}

// =====================================================================================
// 2. dQ kernel (Q-major)
// =====================================================================================
template <int D>
struct DqCfg {
  static constexpr bool kDoResident = D == 256;  // d512: dO streams with V
  static constexpr int kQBytes = D * kTileM * 2;
  static constexpr int kDoBytes = kDoResident ? D * kTileM * 2 : 0;
  static constexpr int kSChunks = D / 128;                    // 128 keys x 128 d
  static constexpr int kPChunks = kDoResident ? D / 128 : D / 64;
  static constexpr int kSmemBytes = kQBytes + kDoBytes + kBwdStages * kStageBytes + kBwdMiscBytes;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmK64,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmDO, const BwdParams p) {
  using Cfg = DqCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_base_ok(smem_raw, p.err)) return;
  uint8_t* smem = smem_raw;
  uint8_t* q_s = smem;
  uint8_t* do_s = smem + Cfg::kQBytes;
  uint8_t* ring = do_s + Cfg::kDoBytes;
  BwdMisc* misc = reinterpret_cast<BwdMisc*>(ring + kBwdStages * kStageBytes);

  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);  // provably warp-uniform
  const int lane = tid & 31;
  const int head = blockIdx.y;
  const int slab = blockIdx.z;
  const int kv_head = head / p.group;

  int seq, qt;
  if (p.q_tiles != nullptr) {
    if (static_cast<int>(blockIdx.x) >= *p.n_q_tiles) return;
    const int2 t = p.q_tiles[blockIdx.x];
    seq = t.x;
    qt = t.y;
  } else {
    const int nqt = (p.layout.seqlen_q + kTileM - 1) / kTileM;
    seq = blockIdx.x / nqt;
    qt = nqt - 1 - static_cast<int>(blockIdx.x % nqt);
  }
  const SeqInfo si = p.layout.seq(seq);
  const int q_off = si.q_off;
  const int64_t tok_base = p.layout.packed() ? si.q_base : static_cast<int64_t>(seq) * p.layout.seqlen_q;

  if (tid == 0) {
    mbar_init(&misc->res_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&misc->ring_full[s], 1);
      mbar_init(&misc->ring_empty[s], 1);
    }
    mbar_init(&misc->s_full, 1);
    mbar_init(&misc->ds_full, kTileM);
    mbar_init(&misc->step_done, 1);
    mbar_init(&misc->drain, 1);
    misc->abort = 0;
    misc->lo = 0x7fffffff;
    misc->hi = -1;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(&misc->tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();

  const int q_idx = qt * kTileM + tid;
  const bool row_valid = tid < kTileM && q_idx < si.len_q;
  const int q_abs = q_idx + q_off;
  const int k_lo = p.mask.window > 0 ? q_abs - p.mask.window + 1 : 0;  // text-only key range start
  int qvis = -1, qdoc = 0;
  float lse2_r = -INFINITY, delta_r = 0.f;
  if (row_valid) {
    if (p.mask.vis) qvis = p.mask.vis[si.meta_base + q_abs];
    if (p.mask.doc) qdoc = p.mask.doc[si.meta_base + q_abs];
    lse2_r = p.lse2[head * p.ws_head_stride + tok_base + q_idx];
    delta_r = p.delta[head * p.ws_head_stride + tok_base + q_idx];
    int lo = p.mask.window > 0 ? max(0, q_abs - p.mask.window + 1) : 0;
    int hi = q_abs;
    if (p.mask.window > 0 && qvis >= 0)
      hi = p.mask.pair_last ? max(hi, p.mask.pair_last[si.meta_base + q_abs]) : si.len_k - 1;
    atomicMin(&misc->lo, lo);
    atomicMax(&misc->hi, min(hi, si.len_k - 1));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = misc->tmem_base;  // S [0,128) dP [128,256) dQ [256,512)
  const int kt_lo = misc->hi >= 0 ? misc->lo / kTileN : 0;
  const int n_kt = misc->hi >= 0 ? misc->hi / kTileN - kt_lo + 1 : 0;
  const CtaAbort ab{&misc->abort, p.err};

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_kt > 0) {
      mbar_expect_tx(&misc->res_full, Cfg::kQBytes + Cfg::kDoBytes);
      for (int blk = 0; blk < D / 64; ++blk)
        tma_load_4d(q_s + blk * 16384, &tmQ, &misc->res_full, blk * 64, head,
                    si.q_base + qt * kTileM, si.b_coord);
      if (Cfg::kDoResident)
        for (int blk = 0; blk < D / 64; ++blk)
          tma_load_4d(do_s + blk * 16384, &tmDO, &misc->res_full, blk * 64, head,
                      si.q_base + qt * kTileM, si.b_coord);
      uint32_t it = 0;
      bool ok = true;
      auto acquire = [&]() -> uint8_t* {
        const uint32_t st = it % kBwdStages;
        const uint32_t ph = (it / kBwdStages) & 1;
        ++it;
        if (!mbar_wait(&misc->ring_empty[st], ph ^ 1, ab, kDevTimeoutMma)) {
          ok = false;
          return nullptr;
        }
        mbar_expect_tx(&misc->ring_full[st], kStageBytes);
        return ring + st * kStageBytes;
      };
      for (int j = 0; j < n_kt && ok; ++j) {
        const int krow = si.k_base + (kt_lo + j) * kTileN;
        for (int c = 0; c < Cfg::kSChunks && ok; ++c) {
          uint8_t* dst = acquire();
          if (!dst) break;
          uint64_t* bar = &misc->ring_full[(it - 1) % kBwdStages];
          for (int h = 0; h < 2; ++h)
            tma_load_4d(dst + h * 16384, &tmK, bar, (2 * c + h) * 64, kv_head, krow, si.b_coord);
        }
        for (int c = 0; c < Cfg::kPChunks && ok; ++c) {
          uint8_t* dst = acquire();
          if (!dst) break;
          uint64_t* bar = &misc->ring_full[(it - 1) % kBwdStages];
          if (Cfg::kDoResident) {
            for (int h = 0; h < 2; ++h)
              tma_load_4d(dst + h * 16384, &tmV, bar, (2 * c + h) * 64, kv_head, krow, si.b_coord);
          } else {
            tma_load_4d(dst, &tmDO, bar, c * 64, head, si.q_base + qt * kTileM, si.b_coord);
            tma_load_4d(dst + 16384, &tmV, bar, c * 64, kv_head, krow, si.b_coord);
          }
        }
        for (int h = 0; h < 2 && ok; ++h) {
          uint8_t* dst = acquire();
          if (!dst) break;
          uint64_t* bar = &misc->ring_full[(it - 1) % kBwdStages];
          for (int blk = 0; blk < 4; ++blk)
            tma_load_4d(dst + blk * 8192, &tmK64, bar, slab * 256 + blk * 64, kv_head,
                        krow + h * 64, si.b_coord);
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    // the whole warp runs the issue loop (warp-uniform waits, one elected
    // lane per MMA): see mbar_wait
    if (n_kt > 0) {
      constexpr uint32_t kIdS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdQ = idesc_bf16(128, 256, false, true);
      const uint32_t qb = smem_addr(q_s);
      const uint32_t db = smem_addr(do_s);
      const uint32_t rb = smem_addr(ring);
      uint32_t it = 0;
      bool ok = mbar_wait(&misc->res_full, 0, ab, kDevTimeoutTma);
      auto take = [&]() -> int {
        const uint32_t st = it % kBwdStages;
        const uint32_t ph = (it / kBwdStages) & 1;
        ++it;
        if (!mbar_wait(&misc->ring_full[st], ph, ab, kDevTimeoutTma)) {
          ok = false;
          return -1;
        }
        tc_fence_after();
        return static_cast<int>(st);
      };
      for (int j = 0; j < n_kt && ok; ++j) {
        // S = Q K^T
        for (int c = 0; c < Cfg::kSChunks && ok; ++c) {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int g = c * 8 + kk;
            umma_ss_w(tmem, sdesc_sw128(qb + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024),
                    sdesc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), kIdS,
                    (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
        }
        // dP = dO V^T
        for (int c = 0; c < Cfg::kPChunks && ok; ++c) {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
          if (Cfg::kDoResident) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const int g = c * 8 + kk;
              umma_ss_w(tmem + 128, sdesc_sw128(db + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024),
                      sdesc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), kIdS,
                      (c | kk) != 0);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_ss_w(tmem + 128, sdesc_sw128(sb + kk * 32, 16, 1024),
                      sdesc_sw128(sb + 16384 + kk * 32, 16, 1024), kIdS, (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
        }
        umma_commit_w(&misc->s_full);
        if (!ok) break;
        if (!(ok = mbar_wait(&misc->ds_full, j & 1, ab, kDevTimeoutPeer))) break;
        tc_fence_after();
        // dQ += dS K   (dS: bf16 pairs in TMEM columns [0,64))
        for (int h = 0; h < 2 && ok; ++h) {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts_w(tmem + 256, tmem + h * 32 + kk * 8, sdesc_sw128(sb + kk * 2048, 8192, 1024),
                    kIdQ, (j | h | kk) != 0);
          umma_commit_w(&misc->ring_empty[st]);
        }
        umma_commit_w(&misc->step_done);
      }
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------- dS warps + epilogue ----------------
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const bool meta = p.mask.has_meta();
    const int qa0 = qt * kTileM + q_off;
    const int qa1 = min((qt + 1) * kTileM, si.len_q) - 1 + q_off;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int k0 = (kt_lo + j) * kTileN;
      const int cls = meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0, si.len_k);
      if (meta) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int kk = k0 + tid;
        const bool in = kk < si.len_k;
        misc->col_vis[tid] = (p.mask.vis && in) ? p.mask.vis[si.meta_base + kk] : -1;
        misc->col_doc[tid] = (p.mask.doc && in) ? p.mask.doc[si.meta_base + kk] : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      if (ok) ok = mbar_wait(&misc->s_full, j & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32], dr[32];
        ld_chunk_pair(lane_base + c * 32, lane_base + 128 + c * 32, sr, dr);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float ds2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c * 32 + i + u;
            const int k = k0 + col;
            bool keep = row_valid && lse2_r != -INFINITY && k < si.len_k;
            if (cls != 1 && keep)  // text only: the key range [k_lo, q_abs]
              keep = meta ? mask_allows(p.mask.window, q_abs, k, qvis, qdoc, misc->col_vis[col],
                                        misc->col_doc[col])
                          : (k >= k_lo && k <= q_abs);
            const float pr = keep ? ex2(fmaf(__uint_as_float(sr[i + u]), kLog2e, -lse2_r)) : 0.f;
            ds2[u] = keep ? pr * (__uint_as_float(dr[i + u]) - delta_r) : 0.f;
          }
          pk[i >> 1] = pack_bf16x2(ds2[0], ds2[1]);
        }
        tmem_st16(lane_base + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&misc->ds_full);
    }
    if (ok && n_kt > 0) ok = mbar_wait(&misc->step_done, (n_kt - 1) & 1, ab, kDevTimeoutMma);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool have = ok && n_kt > 0;
    __nv_bfloat16* dst = p.dq + static_cast<int64_t>(si.b_coord) * p.dq_stride[0] +
                         static_cast<int64_t>(si.q_base + q_idx) * p.dq_stride[1] +
                         static_cast<int64_t>(head) * p.dq_stride[2] + slab * 256;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[32];
      if (have) {
        tmem_ld32(lane_base + 256 + c * 32, r);
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
          out[i] = make_uint4(
              pack_bf16x2(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1])),
              pack_bf16x2(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3])),
              pack_bf16x2(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5])),
              pack_bf16x2(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7])));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_bwd_dq(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tk64,
                  const CUtensorMap& tv, const CUtensorMap& tdo, const BwdParams& p, int grid_x,
                  cudaStream_t stream) {
  using Cfg = DqCfg<D>;
  cudaError_t e = cudaFuncSetAttribute(attn_bwd_dq_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(grid_x, p.num_q_heads, D / 256);
  attn_bwd_dq_kernel<D><<<grid, 192, Cfg::kSmemBytes, stream>>>(tq, tk, tk64, tv, tdo, p);
  return static_cast<int>(cudaGetLastError());
}

// =====================================================================================
// 3. dK/dV kernel (KV-major)
// =====================================================================================
template <int D>
struct DkvCfg {
  static constexpr bool kVResident = D == 256;  // d512: V streams with dO
  static constexpr int kKBytes = D * kTileN * 2;
  static constexpr int kVBytes = kVResident ? D * kTileN * 2 : 0;
  static constexpr int kSChunks = D / 128;
  static constexpr int kPChunks = kVResident ? D / 128 : D / 64;
  static constexpr int kSmemBytes = kKBytes + kVBytes + kBwdStages * kStageBytes + kBwdMiscBytes;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmDO, const BwdParams p) {
  using Cfg = DkvCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_base_ok(smem_raw, p.err)) return;
  uint8_t* smem = smem_raw;
  uint8_t* k_s = smem;
  uint8_t* v_s = smem + Cfg::kKBytes;
  uint8_t* ring = v_s + Cfg::kVBytes;
  BwdMisc* misc = reinterpret_cast<BwdMisc*>(ring + kBwdStages * kStageBytes);

  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);  // provably warp-uniform
  const int lane = tid & 31;
  const int kv_head = blockIdx.y;
  const int slab = blockIdx.z;
  const int G = p.group;

  int seq, kt;
  if (p.k_tiles != nullptr) {
    if (static_cast<int>(blockIdx.x) >= *p.n_k_tiles) return;
    const int2 t = p.k_tiles[blockIdx.x];
    seq = t.x;
    kt = t.y;
  } else {
    const int nkt = (p.layout.seqlen_k + kTileN - 1) / kTileN;
    seq = blockIdx.x / nkt;
    kt = static_cast<int>(blockIdx.x % nkt);
  }
  const SeqInfo si = p.layout.seq(seq);
  const int q_off = si.q_off;
  const int64_t tok_base = p.layout.packed() ? si.q_base : static_cast<int64_t>(seq) * p.layout.seqlen_q;

  if (tid == 0) {
    mbar_init(&misc->res_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&misc->ring_full[s], 1);
      mbar_init(&misc->ring_empty[s], 1);
    }
    mbar_init(&misc->s_full, 1);
    mbar_init(&misc->ds_full, kTileN);
    mbar_init(&misc->step_done, 1);
    mbar_init(&misc->drain, 1);
    misc->abort = 0;
    misc->lo = 0x7fffffff;
    misc->hi = -1;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(&misc->tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();

  // ---- which query positions can see this key tile ----
  const int k = kt * kTileN + tid;  // this thread's key row (tid < 128)
  // text only: the queries that see key k end at k + W - 1 (local) or never
  const int q_hi = p.mask.window > 0
                       ? static_cast<int>(min(static_cast<int64_t>(k) + p.mask.window - 1,
                                              static_cast<int64_t>(0x7fffffff)))
                       : 0x7fffffff;
  const bool row_valid = tid < kTileN && k < si.len_k;
  int kvis = -1, kdoc = 0;
  if (row_valid) {
    if (p.mask.vis) kvis = p.mask.vis[si.meta_base + k];
    if (p.mask.doc) kdoc = p.mask.doc[si.meta_base + k];
    int lo = k;  // causal: q_abs >= k
    if (p.mask.window > 0 && kvis >= 0)
      lo = p.mask.pair_first ? min(lo, p.mask.pair_first[si.meta_base + k]) : 0;
    const int hi = p.mask.window > 0 ? min(si.len_k - 1, k + p.mask.window - 1) : si.len_k - 1;
    atomicMin(&misc->lo, lo);
    atomicMax(&misc->hi, hi);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // query tiles [qt_lo, qt_lo + n_qt) in sequence-local query indices
  int qt_lo = 0, n_qt = 0;
  {
    const int lo_q = max(misc->lo - q_off, 0);
    const int hi_q = min(misc->hi - q_off, si.len_q - 1);
    if (misc->hi >= 0 && hi_q >= lo_q) {
      qt_lo = lo_q / kTileM;
      n_qt = hi_q / kTileM - qt_lo + 1;
    }
  }
  const int n_steps = n_qt * G;
  const uint32_t tmem = misc->tmem_base;  // S^T [0,128) dP^T [128,256) dV [256,384) dK [384,512)
  const CtaAbort ab{&misc->abort, p.err};

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_steps > 0) {
      const int krow = si.k_base + kt * kTileN;
      mbar_expect_tx(&misc->res_full, Cfg::kKBytes + Cfg::kVBytes);
      for (int blk = 0; blk < D / 64; ++blk)
        tma_load_4d(k_s + blk * 16384, &tmK, &misc->res_full, blk * 64, kv_head, krow, si.b_coord);
      if (Cfg::kVResident)
        for (int blk = 0; blk < D / 64; ++blk)
          tma_load_4d(v_s + blk * 16384, &tmV, &misc->res_full, blk * 64, kv_head, krow,
                      si.b_coord);
      uint32_t it = 0;
      bool ok = true;
      auto acquire = [&](uint64_t*& bar) -> uint8_t* {
        const uint32_t st = it % kBwdStages;
        const uint32_t ph = (it / kBwdStages) & 1;
        ++it;
        if (!mbar_wait(&misc->ring_empty[st], ph ^ 1, ab, kDevTimeoutMma)) {
          ok = false;
          return nullptr;
        }
        bar = &misc->ring_full[st];
        mbar_expect_tx(bar, kStageBytes);
        return ring + st * kStageBytes;
      };
      for (int step = 0; step < n_steps && ok; ++step) {
        const int head = kv_head * G + step / n_qt;
        const int qrow = si.q_base + (qt_lo + step % n_qt) * kTileM;
        uint64_t* bar;
        for (int c = 0; c < Cfg::kSChunks && ok; ++c) {
          uint8_t* dst = acquire(bar);
          if (!dst) break;
          for (int h = 0; h < 2; ++h)
            tma_load_4d(dst + h * 16384, &tmQ, bar, (2 * c + h) * 64, head, qrow, si.b_coord);
        }
        for (int c = 0; c < Cfg::kPChunks && ok; ++c) {
          uint8_t* dst = acquire(bar);
          if (!dst) break;
          if (Cfg::kVResident) {
            for (int h = 0; h < 2; ++h)
              tma_load_4d(dst + h * 16384, &tmDO, bar, (2 * c + h) * 64, head, qrow, si.b_coord);
          } else {
            tma_load_4d(dst, &tmV, bar, c * 64, kv_head, krow, si.b_coord);
            tma_load_4d(dst + 16384, &tmDO, bar, c * 64, head, qrow, si.b_coord);
          }
        }
        if (ok) {  // dO slab for dV
          uint8_t* dst = acquire(bar);
          if (dst)
            for (int h = 0; h < 2; ++h)
              tma_load_4d(dst + h * 16384, &tmDO, bar, slab * 128 + h * 64, head, qrow, si.b_coord);
        }
        if (ok) {  // Q slab for dK
          uint8_t* dst = acquire(bar);
          if (dst)
            for (int h = 0; h < 2; ++h)
              tma_load_4d(dst + h * 16384, &tmQ, bar, slab * 128 + h * 64, head, qrow, si.b_coord);
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    // the whole warp runs the issue loop (warp-uniform waits, one elected
    // lane per MMA): see mbar_wait
    if (n_steps > 0) {
      constexpr uint32_t kIdS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdAcc = idesc_bf16(128, 128, false, true);
      const uint32_t kb = smem_addr(k_s);
      const uint32_t vb = smem_addr(v_s);
      const uint32_t rb = smem_addr(ring);
      uint32_t it = 0;
      bool ok = mbar_wait(&misc->res_full, 0, ab, kDevTimeoutTma);
      auto take = [&]() -> int {
        const uint32_t st = it % kBwdStages;
        const uint32_t ph = (it / kBwdStages) & 1;
        ++it;
        if (!mbar_wait(&misc->ring_full[st], ph, ab, kDevTimeoutTma)) {
          ok = false;
          return -1;
        }
        tc_fence_after();
        return static_cast<int>(st);
      };
      for (int step = 0; step < n_steps && ok; ++step) {
        // S^T = K Q^T
        for (int c = 0; c < Cfg::kSChunks && ok; ++c) {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int g = c * 8 + kk;
            umma_ss_w(tmem, sdesc_sw128(kb + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024),
                    sdesc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), kIdS,
                    (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
        }
        // dP^T = V dO^T
        for (int c = 0; c < Cfg::kPChunks && ok; ++c) {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
          if (Cfg::kVResident) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const int g = c * 8 + kk;
              umma_ss_w(tmem + 128, sdesc_sw128(vb + (g >> 2) * 16384 + (g & 3) * 32, 16, 1024),
                      sdesc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), kIdS,
                      (c | kk) != 0);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_ss_w(tmem + 128, sdesc_sw128(sb + kk * 32, 16, 1024),
                      sdesc_sw128(sb + 16384 + kk * 32, 16, 1024), kIdS, (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
        }
        umma_commit_w(&misc->s_full);
        if (!ok) break;
        if (!(ok = mbar_wait(&misc->ds_full, step & 1, ab, kDevTimeoutPeer))) break;
        tc_fence_after();
        // dV += P^T dO[:, slab]
        {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ts_w(tmem + 256, tmem + kk * 8, sdesc_sw128(sb + kk * 2048, 16384, 1024), kIdAcc,
                    (step | kk) != 0);
          umma_commit_w(&misc->ring_empty[st]);
        }
        // dK += dS^T Q[:, slab]
        {
          const int st = take();
          if (st < 0) break;
          const uint32_t sb = rb + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ts_w(tmem + 384, tmem + 128 + kk * 8, sdesc_sw128(sb + kk * 2048, 16384, 1024),
                    kIdAcc, (step | kk) != 0);
          umma_commit_w(&misc->ring_empty[st]);
        }
        umma_commit_w(&misc->step_done);
      }
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------- P^T / dS^T warps + epilogue ----------------
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const bool meta = p.mask.has_meta();
    const int k0 = kt * kTileN;
    bool ok = true;
    for (int step = 0; step < n_steps; ++step) {
      const int head = kv_head * G + step / n_qt;
      const int q0 = (qt_lo + step % n_qt) * kTileM;
      // stage this query tile's LSE / delta / metadata (columns of S^T)
      asm volatile("bar.sync 1, 128;" ::: "memory");
      {
        const int qi = q0 + tid;
        const bool qv = qi < si.len_q;
        misc->col_lse2[tid] = qv ? p.lse2[head * p.ws_head_stride + tok_base + qi] : -INFINITY;
        misc->col_delta[tid] = qv ? p.delta[head * p.ws_head_stride + tok_base + qi] : 0.f;
        if (meta) {
          misc->col_vis[tid] = (p.mask.vis && qv) ? p.mask.vis[si.meta_base + qi + q_off] : -1;
          misc->col_doc[tid] = (p.mask.doc && qv) ? p.mask.doc[si.meta_base + qi + q_off] : 0;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int qa0 = q0 + q_off;
      const int qa1 = min(q0 + kTileM, si.len_q) - 1 + q_off;
      const int cls = meta ? 2 : text_tile_class(p.mask.window, qa0, qa1, k0, si.len_k);
      if (ok) ok = mbar_wait(&misc->s_full, step & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32], dr[32];
        ld_chunk_pair(lane_base + c * 32, lane_base + 128 + c * 32, sr, dr);
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c * 32 + i + u;
            const float l2 = misc->col_lse2[col];
            bool keep = row_valid && l2 != -INFINITY;
            if (cls != 1 && keep)  // text only: the query range [k, q_hi]
              keep = meta ? mask_allows(p.mask.window, q0 + col + q_off, k, misc->col_vis[col],
                                        misc->col_doc[col], kvis, kdoc)
                          : (q0 + col + q_off >= k && q0 + col + q_off <= q_hi);
            const float pr = keep ? ex2(fmaf(__uint_as_float(sr[i + u]), kLog2e, -l2)) : 0.f;
            pv[u] = pr;
            dv[u] = keep ? pr * (__uint_as_float(dr[i + u]) - misc->col_delta[col]) : 0.f;
          }
          pp[i >> 1] = pack_bf16x2(pv[0], pv[1]);
          pd[i >> 1] = pack_bf16x2(dv[0], dv[1]);
        }
        tmem_st16(lane_base + c * 16, pp);
        tmem_st16(lane_base + 128 + c * 16, pd);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&misc->ds_full);
    }
    if (ok && n_steps > 0) ok = mbar_wait(&misc->step_done, (n_steps - 1) & 1, ab, kDevTimeoutMma);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool have = ok && n_steps > 0;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {  // 0: dV, 1: dK
      __nv_bfloat16* base = which == 0 ? p.dv : p.dk;
      const int64_t* stv = which == 0 ? p.dv_stride : p.dk_stride;
      __nv_bfloat16* dst = base + static_cast<int64_t>(si.b_coord) * stv[0] +
                           static_cast<int64_t>(si.k_base + k) * stv[1] +
                           static_cast<int64_t>(kv_head) * stv[2] + slab * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        if (have) {
          tmem_ld32(lane_base + 256 + which * 128 + c * 32, r);
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
            out[i] = make_uint4(
                pack_bf16x2(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1])),
                pack_bf16x2(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3])),
                pack_bf16x2(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5])),
                pack_bf16x2(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7])));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_bwd_dkv(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const CUtensorMap& tdo, const BwdParams& p, int grid_x, cudaStream_t stream) {
  using Cfg = DkvCfg<D>;
  cudaError_t e = cudaFuncSetAttribute(attn_bwd_dkv_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(grid_x, p.num_q_heads / p.group, D / 128);
  attn_bwd_dkv_kernel<D><<<grid, 192, Cfg::kSmemBytes, stream>>>(tq, tk, tv, tdo, p);
  return static_cast<int>(cudaGetLastError());
}

template int launch_bwd_dq<256>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                const CUtensorMap&, const CUtensorMap&, const BwdParams&, int,
                                cudaStream_t);
template int launch_bwd_dq<512>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                const CUtensorMap&, const CUtensorMap&, const BwdParams&, int,
                                cudaStream_t);
template int launch_bwd_dkv<256>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                 const CUtensorMap&, const BwdParams&, int, cudaStream_t);
template int launch_bwd_dkv<512>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                 const CUtensorMap&, const BwdParams&, int, cudaStream_t);

}  // namespace g4
