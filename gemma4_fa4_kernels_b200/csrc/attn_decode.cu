// Single-token decode against a KV cache for sm_100a: one query token per
// sequence (fixed layout Sq == 1, or packed segments with at most one query)
// reading the whole allowed key range of its cache once.  HBM-bound: the K/V
// bytes of the active range dominate everything else.
//
// Work split: CTA (split, kv head, sequence) takes a contiguous run of
// 128-key tiles of that KV head and serves all `group` query heads that share
// it, so every K/V byte crosses HBM exactly once.  The contraction runs
// transposed on the tensor core so the few query heads sit on the narrow
// N = 16 side of a 128 x 16 MMA instead of wasting a 128-row M:
//   S^T (128 keys x 16 heads)  = K_tile (128 x D)  . Q^T (D x 16)       [TMEM]
//   O^T (D x 16 heads)        += V_tile^T (D x 128) . P^T (128 x 16)   [TMEM, D/128 MMAs of M=128]
// K and V tiles stream through a ring of 32 KB shared-memory stages (128 keys x
// 128 head-dim elements, two 128-B-swizzled TMA boxes) in MMA order
// K(0), K(1), V(0), K(2), V(1), ...; the V stages serve directly as the
// MN-major A operand of the O^T MMA.  Q^T and P^T are staged by ordinary
// stores in the K-major swizzled layout (rows = heads, zero-padded to 16).
//
// Warp roles (192 threads): warps 0-3 softmax (thread i = key i of the tile =
// TMEM lane i; per-head maxima and sums are reduced across the 128 threads),
// warp 4 TMA producer + TMEM owner, warp 5 MMA issuer.  Online softmax in the
// exp2 domain with the same lazy rescale rule as the prefill kernels.  With
// more than one split per (sequence, KV head) every CTA writes its unnormalised
// O, running max and row sum, and decode_combine_kernel merges them.
//
// Mask for a single query at the lower-right position q = Sk - 1: every key is
// causal, so the vision rule never changes the answer; the local window keeps
// keys k > q - W and documents keep doc[k] == doc[q] (masks.py:8-80).
//
// Reference interface replaced: the attention inside the static-cache decode
// ops (src/gemma4_fa4/h100_torch_ops.py:692-880), which route one query token
// through fa4_local_varlen_forward / fa4_global_text_forward (query padded to
// the cache length) / fa4_global_forward_only.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "g4_attn.cuh"
#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

namespace {

constexpr int kStageBytes = 32768;
constexpr int kPBufBytes = 4096;  // 16 heads x 128 keys bf16, two 64-key slabs

struct DecMisc {
  uint64_t ring_full[kDecodeStages];
  uint64_t ring_empty[kDecodeStages];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full[2];
  uint64_t p_free[2];
  uint64_t drain;
  uint64_t q_ready;
  uint32_t tmem_base;
  int abort;
  float red[2][4][16];  // per-tile maxima of each warp (double-buffered)
  float red_l[4][16];
};
static_assert(sizeof(DecMisc) <= 1024, "decode misc block exceeds its reservation");

template <int D>
struct DecCfg {
  static constexpr int kChunks = D / 128;  // ring stages per K (or V) tile
  static constexpr int kQBytes = (D / 64) * 2048;
  static constexpr int kSmemBytes =
      kDecodeStages * kStageBytes + kQBytes + 2 * kPBufBytes + 1024 /*misc*/ + 1024 /*align*/;
};

// TMEM columns: S^T buffers [0,16) and [16,32); O^T chunk c at 32 + 16c.
constexpr uint32_t kTmemCols = 128;

__device__ __forceinline__ void named_bar_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

}  // namespace

template <int D>
__global__ void __launch_bounds__(192, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const DecodeParams p) {
  using Cfg = DecCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* q_s = ring + kDecodeStages * kStageBytes;
  uint8_t* p_s = q_s + Cfg::kQBytes;
  DecMisc* misc = reinterpret_cast<DecMisc*>(p_s + 2 * kPBufBytes);

  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0);  // provably warp-uniform
  const int lane = tid & 31;
  const int split = blockIdx.x;
  const int kv_head = blockIdx.y;
  const int seq = blockIdx.z;
  const SeqInfo si = p.layout.seq(seq);
  if (si.len_q <= 0) return;  // packed segment without a query token (whole CTA)

  const int G = p.group;
  const int head0 = kv_head * G;
  const int q_abs = si.len_k - 1;
  const int k_lo = p.window > 0 ? max(0, q_abs - p.window + 1) : 0;
  const int n_tiles = si.len_k > 0 ? (si.len_k - k_lo + kTileN - 1) / kTileN : 0;
  const int tps = (n_tiles + p.n_split - 1) / p.n_split;
  const int t_begin = split * tps;
  const int n = max(0, min(n_tiles, t_begin + tps) - t_begin);

  if (tid == 0) {
    for (int s = 0; s < kDecodeStages; ++s) {
      mbar_init(&misc->ring_full[s], 1);
      mbar_init(&misc->ring_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&misc->s_full[b], 1);
      mbar_init(&misc->s_empty[b], kTileN);
      mbar_init(&misc->p_full[b], kTileN);
      mbar_init(&misc->p_free[b], 1);
    }
    mbar_init(&misc->drain, 1);
    mbar_init(&misc->q_ready, kTileN);
    misc->abort = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(&misc->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The merge kernel is launched as a programmatic dependent: let it start
  // now; it waits for this grid's completion before reading anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const uint32_t tmem = misc->tmem_base;
  const CtaAbort ab{&misc->abort, p.err};

  if (warp == 4) {
    // ============================ TMA producer ============================
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t it = 0;
      bool ok = true;
      // Each K (or V) tile claims all of its ring stages before any of its
      // boxes is issued, so the whole 1 KB cache rows of a tile reach DRAM as
      // one burst (measured ~4% faster than issuing stage by stage).
      auto load = [&](const CUtensorMap* map, int u) {
        const int tok = si.k_base + k_lo + (t_begin + u) * kTileN;
        for (int c = 0; c < Cfg::kChunks && ok; ++c) {
          const uint32_t st = (it + c) % kDecodeStages;
          const uint32_t ph = ((it + c) / kDecodeStages) & 1;
          ok = mbar_wait(&misc->ring_empty[st], ph ^ 1, ab, kDevTimeoutMma);
        }
        if (!ok) return;
        for (int c = 0; c < Cfg::kChunks; ++c) {
          const uint32_t st = (it + c) % kDecodeStages;
          mbar_expect_tx(&misc->ring_full[st], kStageBytes);
          for (int h = 0; h < 2; ++h)
            tma_load_4d(ring + st * kStageBytes + h * 16384, map, &misc->ring_full[st],
                        c * 128 + h * 64, kv_head, tok, si.b_coord);
        }
        it += Cfg::kChunks;
      };
      load(&tmK, 0);
      for (int u = 0; u < n && ok; ++u) {
        if (u + 1 < n) load(&tmK, u + 1);
        load(&tmV, u);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ============================ MMA issuer ============================
    // the whole warp runs the issue loop (warp-uniform waits, one elected
    // lane per MMA): see mbar_wait
    if (n > 0) {
      constexpr uint32_t kIdS = idesc_bf16(128, 16, false, false);
      constexpr uint32_t kIdO = idesc_bf16(128, 16, true, false);
      const uint32_t ring_b = smem_addr(ring);
      const uint32_t q_b = smem_addr(q_s);
      const uint32_t p_b = smem_addr(p_s);
      uint32_t it = 0;
      bool ok = mbar_wait(&misc->q_ready, 0, ab, kDevTimeoutPeer);
      auto take = [&](uint32_t& stage) -> bool {
        stage = it % kDecodeStages;
        const uint32_t ph = (it / kDecodeStages) & 1;
        if (!mbar_wait(&misc->ring_full[stage], ph, ab, kDevTimeoutTma)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int u) {
        const int b = u & 1;
        if (!(ok = mbar_wait(&misc->s_empty[b], ((u >> 1) & 1) ^ 1, ab, kDevTimeoutPeer)))
          return;
        tc_fence_after();
        const uint32_t d = tmem + b * 16;
        for (int c = 0; c < Cfg::kChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = take(st))) break;
          const uint32_t kb = ring_b + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = sdesc_sw128(kb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t bq =
                sdesc_sw128(q_b + (2 * c + (kk >> 2)) * 2048 + (kk & 3) * 32, 16, 1024);
            umma_ss_w(d, a, bq, kIdS, (c | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
          ++it;
        }
        umma_commit_w(&misc->s_full[b]);
      };
      auto issue_o = [&](int u) {
        const int b = u & 1;
        for (int c = 0; c < Cfg::kChunks && ok; ++c) {
          uint32_t st;
          if (!(ok = take(st))) break;
          const uint32_t vb = ring_b + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = sdesc_sw128(vb + kk * 2048, 16384, 1024);
            const uint64_t bp =
                sdesc_sw128(p_b + b * kPBufBytes + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024);
            umma_ss_w(tmem + 32 + c * 16, a, bp, kIdO, (u | kk) != 0);
          }
          umma_commit_w(&misc->ring_empty[st]);
          ++it;
        }
        umma_commit_w(&misc->p_free[b]);
      };
      if (ok) issue_s(0);
      for (int u = 0; u < n && ok; ++u) {
        if (u + 1 < n) issue_s(u + 1);
        if (!ok) break;
        if (!(ok = mbar_wait(&misc->p_full[u & 1], (u >> 1) & 1, ab, kDevTimeoutPeer)))
          break;
        tc_fence_after();
        issue_o(u);
      }
      // Drain: every MMA this warp issued has completed before TMEM is freed.
      umma_commit_w(&misc->drain);
      mbar_wait(&misc->drain, 0, ab, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ===================== softmax + epilogue (warps 0-3) =====================
    // tcgen05.ld/st are .sync.aligned: control flow around them stays
    // warp-uniform (`ok` is reduced with __all_sync; the rescale decision is
    // identical in every thread because it depends on CTA-wide maxima only).
    // Q^T: rows = the group's query heads (zero rows up to 16), 64 head-dim
    // elements per 128-B row, one 2 KB slab per 64 elements, 128-B swizzle.
    // Staged while the producer's first K loads are already in flight.
    {
      const __nv_bfloat16* qb = p.q + static_cast<int64_t>(si.b_coord) * p.q_stride[0] +
                                static_cast<int64_t>(si.q_base) * p.q_stride[1];
      constexpr int kRowChunks = D / 8;
      for (int idx = tid; idx < 16 * kRowChunks; idx += 128) {
        const int row = idx / kRowChunks;
        const int cg = idx % kRowChunks;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < G)
          v = *reinterpret_cast<const uint4*>(
              qb + static_cast<int64_t>(head0 + row) * p.q_stride[2] + cg * 8);
        *reinterpret_cast<uint4*>(q_s + (cg >> 3) * 2048 + row * 128 +
                                  (((cg & 7) ^ (row & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&misc->q_ready);
    }
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_run[16], l_part[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      m_run[j] = -INFINITY;
      l_part[j] = 0.f;
    }
    const int qdoc = (p.doc != nullptr && si.len_k > 0) ? p.doc[si.meta_base + q_abs] : 0;
    bool ok = true;
    for (int u = 0; u < n; ++u) {
      const int b = u & 1;
      const int k = k_lo + (t_begin + u) * kTileN + tid;
      bool valid = k < si.len_k;
      if (valid && p.doc != nullptr) valid = p.doc[si.meta_base + k] == qdoc;
      if (ok) ok = mbar_wait(&misc->s_full[b], (u >> 1) & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      float s[16];
      if (ok) {
        tc_fence_after();
        uint32_t r[16];
        tmem_ld16(lane_base + b * 16, r);
        tmem_wait_ld();
        reg_fence16(r);
#pragma unroll
        for (int j = 0; j < 16; ++j) s[j] = valid ? __uint_as_float(r[j]) * kLog2e : -INFINITY;
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) s[j] = -INFINITY;
      }
      tc_fence_before();
      if (ok) mbar_arrive(&misc->s_empty[b]);

      // per-head maximum over the tile's 128 keys
      float mt[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float v = s[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        mt[j] = v;
      }
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) misc->red[b][warp][j] = mt[j];
      }
      named_bar_softmax();
#pragma unroll
      for (int j = 0; j < 16; ++j)
        mt[j] = fmaxf(fmaxf(misc->red[b][0][j], misc->red[b][1][j]),
                      fmaxf(misc->red[b][2][j], misc->red[b][3][j]));
      bool rescale = false;
      float alpha[16], pv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        alpha[j] = 1.f;
        if (mt[j] > m_run[j] + kLazyRescaleLog2) {  // also the first finite tile
          // a head without any finite score so far has O = 0 and l = 0
          if (m_run[j] != -INFINITY) {
            alpha[j] = ex2(m_run[j] - mt[j]);
            rescale = true;
          }
          m_run[j] = mt[j];
        }
        const float m_sub = (m_run[j] == -INFINITY) ? 0.f : m_run[j];
        pv[j] = ex2(s[j] - m_sub);
        l_part[j] = l_part[j] * alpha[j] + pv[j];
      }

      // P^T(u) into its buffer once the O^T MMAs of tile u-2 have read it
      if (ok) ok = mbar_wait(&misc->p_free[b], ((u >> 1) & 1) ^ 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
      {
        uint8_t* pb = p_s + b * kPBufBytes + (tid >> 6) * 2048;
        const int kc = (tid & 63) >> 3;
        const int ke = (tid & 7) * 2;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          *reinterpret_cast<__nv_bfloat16*>(pb + j * 128 + ((kc ^ (j & 7)) << 4) + ke) =
              __float2bfloat16_rn(pv[j]);
      }
      if (rescale && u > 0) {
        // O^T must hold every earlier tile before it is scaled in place.
        if (ok) ok = mbar_wait(&misc->p_free[(u - 1) & 1], ((u - 1) >> 1) & 1, ab, kDevTimeoutMma);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < Cfg::kChunks; ++c) {
            uint32_t r[16];
            tmem_ld16(lane_base + 32 + c * 16, r);
            tmem_wait_ld();
            reg_fence16(r);
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha[j]);
            tmem_st16(lane_base + 32 + c * 16, r);
          }
          tmem_wait_st();
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (ok) mbar_arrive(&misc->p_full[b]);
    }

    // ---- epilogue ----
    if (n > 0) {
      if (ok) ok = mbar_wait(&misc->p_free[(n - 1) & 1], ((n - 1) >> 1) & 1, ab, kDevTimeoutMma);
      ok = __all_sync(0xffffffffu, ok);
    }
    tc_fence_after();
    float L[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = l_part[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      L[j] = v;
    }
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) misc->red_l[warp][j] = L[j];
    }
    named_bar_softmax();
#pragma unroll
    for (int j = 0; j < 16; ++j)
      L[j] = (misc->red_l[0][j] + misc->red_l[1][j]) + (misc->red_l[2][j] + misc->red_l[3][j]);
    const bool have_o = ok && n > 0;
    if (p.n_split == 1) {
      __nv_bfloat16* ob = p.o + static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
                          static_cast<int64_t>(si.q_base) * p.o_stride[1];
#pragma unroll 1
      for (int c = 0; c < Cfg::kChunks; ++c) {
        uint32_t r[16];
        if (have_o) {
          tmem_ld16(lane_base + 32 + c * 16, r);
          tmem_wait_ld();
          reg_fence16(r);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (j < G) {
            const float inv = L[j] > 0.f ? 1.f / L[j] : 0.f;
            ob[static_cast<int64_t>(head0 + j) * p.o_stride[2] + c * 128 + tid] =
                __float2bfloat16_rn(__uint_as_float(r[j]) * inv);
          }
        }
      }
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (j < G) {
            const float lse = (have_o && L[j] > 0.f) ? (m_run[j] + __log2f(L[j])) * kLn2 : -INFINITY;
            p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
                  static_cast<int64_t>(head0 + j) * p.lse_stride[1] + si.q_base] = lse;
          }
        }
      }
    } else {
      const int64_t base = (static_cast<int64_t>(seq) * p.num_q_heads + head0) * p.n_split + split;
      // written even without keys (zeros), so the merge never reads stale data
#pragma unroll 1
      for (int c = 0; c < Cfg::kChunks; ++c) {
        uint32_t r[16];
        if (have_o) {
          tmem_ld16(lane_base + 32 + c * 16, r);
          tmem_wait_ld();
          reg_fence16(r);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < G)
            p.part_o[(base + static_cast<int64_t>(j) * p.n_split) * D + c * 128 + tid] =
                __uint_as_float(r[j]);
      }
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < G)
            p.part_ml[base + static_cast<int64_t>(j) * p.n_split] =
                make_float2(m_run[j], have_o ? L[j] : 0.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge the key-range splits of one (sequence, query head), one thread per
// head-dim element (grid: D/128 x Hq x sequences):
//   M = max m_x,  w_x = 2^(m_x - M),  O = sum w_x O_x / sum w_x l_x,
//   LSE = (M + log2 sum w_x l_x) ln 2; splits with l_x = 0 get w_x = 0.
// Every partial-O load of a batch of kMergeBatch splits is issued before the
// split statistics are reduced, so one memory round trip serves the batch.
// Launched as a programmatic dependent of decode_kernel: griddepcontrol.wait
// returns once that grid has completed and its writes are visible.
constexpr int kMergeBatch = 48;

template <int D>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeParams p) {
  __shared__ float m_s[kMergeBatch];
  __shared__ float l_s[kMergeBatch];
  __shared__ float red[4];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int head = blockIdx.y;
  const int seq = blockIdx.z;
  const int tid = threadIdx.x;
  const int d = blockIdx.x * 128 + tid;
  const SeqInfo si = p.layout.seq(seq);
  if (si.len_q <= 0) return;
  const int ns = p.n_split;
  const int64_t base = (static_cast<int64_t>(seq) * p.num_q_heads + head) * ns;
  const float* po = p.part_o + base * D + d;
  float M = -INFINITY, L = 0.f, acc = 0.f;  // running merge across batches
  for (int x0 = 0; x0 < ns; x0 += kMergeBatch) {
    const int nb = min(kMergeBatch, ns - x0);
    float o[kMergeBatch];
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i)
      o[i] = i < nb ? po[static_cast<int64_t>(x0 + i) * D] : 0.f;
    float mloc = -INFINITY;
    if (tid < nb) {
      const float2 v = p.part_ml[base + x0 + tid];
      m_s[tid] = v.x;
      l_s[tid] = v.y;
      if (v.y > 0.f) mloc = v.x;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
    if ((tid & 31) == 0) red[tid >> 5] = mloc;
    __syncthreads();
    const float mb = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float m_new = fmaxf(M, mb);
    if (m_new != -INFINITY) {
      const float scale = M == -INFINITY ? 0.f : ex2(M - m_new);
      L *= scale;
      acc *= scale;
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        if (i < nb && l_s[i] > 0.f) {
          const float w = ex2(m_s[i] - m_new);
          L = fmaf(w, l_s[i], L);
          acc = fmaf(w, o[i], acc);
        }
      }
      M = m_new;
    }
    __syncthreads();
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  p.o[static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
      static_cast<int64_t>(si.q_base) * p.o_stride[1] + static_cast<int64_t>(head) * p.o_stride[2] +
      d] = __float2bfloat16_rn(acc * inv);
  if (blockIdx.x == 0 && tid == 0)
    p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
          static_cast<int64_t>(head) * p.lse_stride[1] + si.q_base] =
        L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
}

int decode_smem_bytes(int d) {
  return d == 256 ? DecCfg<256>::kSmemBytes : DecCfg<512>::kSmemBytes;
}

int launch_decode(int d, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                  int num_kv_heads, cudaStream_t stream) {
  const dim3 grid(p.n_split, num_kv_heads, p.layout.batch);
  cudaError_t e;
  if (d == 256) {
    e = cudaFuncSetAttribute(decode_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<256>::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    decode_kernel<256><<<grid, 192, DecCfg<256>::kSmemBytes, stream>>>(tk, tv, p);
  } else {
    e = cudaFuncSetAttribute(decode_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<512>::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    decode_kernel<512><<<grid, 192, DecCfg<512>::kSmemBytes, stream>>>(tk, tv, p);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_decode_combine(int d, const DecodeParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(d / 128, p.num_q_heads, p.layout.batch);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = d == 256 ? cudaLaunchKernelEx(&cfg, decode_combine_kernel<256>, p)
                           : cudaLaunchKernelEx(&cfg, decode_combine_kernel<512>, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4
