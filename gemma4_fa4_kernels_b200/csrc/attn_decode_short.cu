// Single-token decode against a short key range (sliding-window layers) for
// sm_100a, on the CUDA cores, in one launch.
//
// A decode call against a 1024-token window reads 16.8 MB (32Q/16KV, d256):
// about 2.6 us of HBM time.  At that size the tensor-core decode kernel's fixed
// costs (TMEM allocation, barrier set-up, the ring's first fill) and the
// separate merge launch dominate.  Here every CTA streams its slice of keys
// with 16-byte loads and does the few dot products per key on the CUDA cores
// (a query group of at most 4 heads gives 2 FLOP per K/V byte), so a CTA is
// busy from its first instruction.
//
// CTA (split, KV head, sequence), 256 threads, at most decode_short_keys(D, G)
// keys (64 for d256 with groups of up to 2 heads: 32 KB of K and V).  Every
// warp works alone on its own keys until the CTA combine:
//   1. the warp requests its K rows, V rows (this lane's D/32 features of each)
//      and the group's query features up front, so the whole slice is in
//      flight at once;
//   2. scores: per key and head a lane's partial dot product, summed by xor
//      shuffles (every lane ends with every score); masked keys get -inf;
//   3. the warp's softmax over its keys (exp2 domain, as the other kernels) and
//      its unnormalised O = sum p V, all in registers;
//   4. the warps' (max, sum, O) are combined through shared memory.
// One split writes O and LSE directly.  With several splits each CTA writes its
// unnormalised O, max and sum, then takes a ticket on the (sequence, KV head)
// counter; the CTA that takes the last ticket merges every split (exact
// log-sum-exp combination, every split's partial requested at once) and resets
// the counter for the next call.
//
// Mask for the single query at q = Sk - 1: every key is causal (the vision rule
// never adds a key), the window keeps k > q - W and documents doc[k] == doc[q]
// (masks.py:8-80).  Replaces the same attention as attn_decode.cu (the
// static-cache decode ops, h100_torch_ops.py:692-880).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_attn.cuh"
#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {

namespace {

constexpr int kShortThreads = 256;
constexpr int kShortWarps = kShortThreads / 32;

__device__ __forceinline__ void bf16x8_to_float(const uint4& w, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

template <int D, int G>
struct ShortCfg {
  static constexpr int kPerLane = D / 32;                // features of a row per lane
  static constexpr int kLoads = kPerLane / 8;            // 16-B loads per lane and row
  static constexpr int kKeys = decode_short_keys(D, G);  // keys per CTA at most
  static constexpr int kKeysPerWarp = kKeys / kShortWarps;
  static constexpr int kOut = G * D / kShortThreads;     // combined outputs per thread
  // merge: split partials requested per batch and output (one batch covers the
  // 18 splits of a 16-KV-head d256 cache with groups of up to two heads)
  static constexpr int kBatch = kOut >= 8 ? 4 : 40 / kOut;
  // warp partials: O [warp][G][D], max and sum [warp][G]
  static constexpr int kSmemBytes = (kShortWarps * G * D + 2 * kShortWarps * G) * 4;
  static_assert(kKeysPerWarp >= 1 && kKeys == kKeysPerWarp * kShortWarps, "keys per warp");
  static_assert(G * D % kShortThreads == 0, "outputs per thread");
  // the merge keeps each split's weight and sum in the warp partials' space
  static_assert(2 * kDecodeShortMaxSplits <= kShortWarps * D, "merge scratch fits");
};

}  // namespace

template <int D, int G>
__global__ void __launch_bounds__(kShortThreads, 2) decode_short_kernel(const DecodeParams p) {
  using Cfg = ShortCfg<D, G>;
  constexpr int kPerLane = Cfg::kPerLane, kLoads = Cfg::kLoads, kKPW = Cfg::kKeysPerWarp;
  extern __shared__ __align__(16) float sm[];
  float* wo = sm;                                   // [warp][G][D]
  float* wm = wo + kShortWarps * G * D;             // [warp][G]
  float* wl = wm + kShortWarps * G;                 // [warp][G]
  __shared__ int last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const SeqInfo si = p.layout.seq(seq);
  if (si.len_q <= 0) {  // packed segment without a query token (whole CTA)
    pdl_enter();  // every exit waits: the grid's completion implies the reset's
    return;
  }
  const int q_abs = si.len_k - 1;
  const int k_lo = p.window > 0 ? max(0, q_abs - p.window + 1) : 0;
  const int total = max(0, si.len_k - k_lo);
  const int per = (total + p.n_split - 1) / p.n_split;
  const int kb = k_lo + split * per;
  const int n = min(Cfg::kKeys, max(0, min(si.len_k, kb + per) - kb));
  const int head0 = kvh * G;
  const int j0 = warp * kKPW;  // this warp's first key in the CTA's slice

  // ---- 1. every load of the warp in flight at once ----
  const __nv_bfloat16* kbase = p.k + static_cast<int64_t>(si.b_coord) * p.k_stride[0] +
                               static_cast<int64_t>(kvh) * p.k_stride[2] + lane * 8;
  const __nv_bfloat16* vbase = p.v + static_cast<int64_t>(si.b_coord) * p.v_stride[0] +
                               static_cast<int64_t>(kvh) * p.v_stride[2] + lane * 8;
  uint4 kr[kKPW][kLoads], vr[kKPW][kLoads];
#pragma unroll
  for (int i = 0; i < kKPW; ++i) {
    const bool in = j0 + i < n;
    const int64_t t = si.k_base + kb + min(j0 + i, max(n - 1, 0));
#pragma unroll
    for (int l = 0; l < kLoads; ++l) {
      kr[i][l] = in ? *reinterpret_cast<const uint4*>(kbase + t * p.k_stride[1] + l * 256)
                    : make_uint4(0, 0, 0, 0);
      vr[i][l] = in ? *reinterpret_cast<const uint4*>(vbase + t * p.v_stride[1] + l * 256)
                    : make_uint4(0, 0, 0, 0);
    }
  }
  uint4 qr[G][kLoads];
  const __nv_bfloat16* qbase = p.q + static_cast<int64_t>(si.b_coord) * p.q_stride[0] +
                               static_cast<int64_t>(si.q_base) * p.q_stride[1] + lane * 8;
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int l = 0; l < kLoads; ++l)
      qr[h][l] = *reinterpret_cast<const uint4*>(
          qbase + static_cast<int64_t>(head0 + h) * p.q_stride[2] + l * 256);
  int kdoc[kKPW];
  int qdoc = 0;
  if (p.doc != nullptr) {
    qdoc = p.doc[si.meta_base + q_abs];
#pragma unroll
    for (int i = 0; i < kKPW; ++i) kdoc[i] = j0 + i < n ? p.doc[si.meta_base + kb + j0 + i] : 0;
  }

  // ---- 2. scores (log2 domain), summed across the warp ----
  float s[G][kKPW];
  {
    float qf[G][kPerLane];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int l = 0; l < kLoads; ++l) bf16x8_to_float(qr[h][l], qf[h] + l * 8);
#pragma unroll
    for (int i = 0; i < kKPW; ++i) {
      float kf[kPerLane];
#pragma unroll
      for (int l = 0; l < kLoads; ++l) bf16x8_to_float(kr[i][l], kf + l * 8);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < kPerLane; ++e) acc = fmaf(qf[h][e], kf[e], acc);
        s[h][i] = acc;
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < kKPW; ++i) s[h][i] += __shfl_xor_sync(0xffffffffu, s[h][i], off);

  // ---- 3. the warp's softmax and O over its keys ----
  float m[G], l[G], acc[G][kPerLane];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
#pragma unroll
    for (int i = 0; i < kKPW; ++i) {
      const bool keep = j0 + i < n && (p.doc == nullptr || kdoc[i] == qdoc);
      s[h][i] = keep ? s[h][i] * kLog2e : -INFINITY;
      m[h] = fmaxf(m[h], s[h][i]);
    }
    const float msub = m[h] == -INFINITY ? 0.f : m[h];
    l[h] = 0.f;
#pragma unroll
    for (int i = 0; i < kKPW; ++i) {
      s[h][i] = ex2(s[h][i] - msub);  // exp2(-inf) = 0
      l[h] += s[h][i];
    }
#pragma unroll
    for (int e = 0; e < kPerLane; ++e) acc[h][e] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < kKPW; ++i) {
    float vf[kPerLane];
#pragma unroll
    for (int q = 0; q < kLoads; ++q) bf16x8_to_float(vr[i][q], vf + q * 8);
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < kPerLane; ++e) acc[h][e] = fmaf(s[h][i], vf[e], acc[h][e]);
  }

  // ---- 4. combine the warps ----
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float* dst = wo + (warp * G + h) * D + lane * 8;
#pragma unroll
    for (int q = 0; q < kLoads; ++q) {
      reinterpret_cast<float4*>(dst + q * 256)[0] =
          make_float4(acc[h][q * 8 + 0], acc[h][q * 8 + 1], acc[h][q * 8 + 2], acc[h][q * 8 + 3]);
      reinterpret_cast<float4*>(dst + q * 256)[1] =
          make_float4(acc[h][q * 8 + 4], acc[h][q * 8 + 5], acc[h][q * 8 + 6], acc[h][q * 8 + 7]);
    }
    if (lane == 0) {
      wm[warp * G + h] = m[h];
      wl[warp * G + h] = l[h];
    }
  }
  __syncthreads();
  const int ns = p.n_split;
  const int hq = p.num_q_heads;
  float co[Cfg::kOut], cm[Cfg::kOut], cl[Cfg::kOut];  // this CTA's O, max and sum
#pragma unroll
  for (int c = 0; c < Cfg::kOut; ++c) {
    const int i = tid + c * kShortThreads;
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kShortWarps; ++w)
      if (wl[w * G + h] > 0.f) M = fmaxf(M, wm[w * G + h]);
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < kShortWarps; ++w) {
      const float lw = wl[w * G + h];
      const float x = lw > 0.f ? ex2(wm[w * G + h] - M) : 0.f;
      L = fmaf(x, lw, L);
      o = fmaf(x, wo[(w * G + h) * D + d], o);
    }
    co[c] = o;
    cm[c] = M;
    cl[c] = L;
  }
  if (ns == 1) {
#pragma unroll
    for (int c = 0; c < Cfg::kOut; ++c) {
      const int i = tid + c * kShortThreads;
      const int h = i / D, d = i % D;
      p.o[static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
          static_cast<int64_t>(si.q_base) * p.o_stride[1] +
          static_cast<int64_t>(head0 + h) * p.o_stride[2] + d] =
          __float2bfloat16_rn(cl[c] > 0.f ? co[c] / cl[c] : 0.f);
      if (d == 0)
        p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
              static_cast<int64_t>(head0 + h) * p.lse_stride[1] + si.q_base] =
            cl[c] > 0.f ? (cm[c] + __log2f(cl[c])) * kLn2 : -INFINITY;
    }
    pdl_enter();
    return;
  }

  // ---- several splits: partials, then the last arriving CTA merges ----
#pragma unroll
  for (int c = 0; c < Cfg::kOut; ++c) {
    const int i = tid + c * kShortThreads;
    const int h = i / D, d = i % D;
    const int64_t row = (static_cast<int64_t>(seq) * hq + head0 + h) * ns + split;
    p.part_o[row * D + d] = co[c];
    if (d == 0) p.part_ml[row] = make_float2(cm[c], cl[c]);
  }
  // Release and acquire through one thread (the pattern of a grid-wide
  // barrier): the CTA barrier orders every thread's partial stores before
  // thread 0's fence and ticket; in the CTA that takes the last ticket, thread
  // 0's fence after it orders every split's partials before the barrier that
  // releases the merge's loads.
  __syncthreads();
  // The counters were zeroed by the call's workspace reset kernel, which let
  // this grid launch at once: everything above ran under it, the first counter
  // access waits for it.
  pdl_enter();
  int* counter = p.counters + static_cast<int64_t>(seq) * gridDim.y + kvh;
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(counter, 1) == ns - 1;
    if (last) __threadfence();
  }
  __syncthreads();
  if (!last) return;
  // Merge: every thread requests its outputs' first batch of split partials
  // and warps < G the splits' (max, sum) at once; then per head the weights
  // 2^(m_s - M) / L (warp h, in shared memory over the warp partials, which are
  // no longer read), and every thread sums its outputs over the splits.
  float v[Cfg::kOut][Cfg::kBatch];
  auto load_batch = [&](int s0) {
#pragma unroll
    for (int c = 0; c < Cfg::kOut; ++c) {
      const int i = tid + c * kShortThreads;
      const int h = i / D, d = i % D;
      const float* po = p.part_o + (static_cast<int64_t>(seq) * hq + head0 + h) * ns * D + d;
#pragma unroll
      for (int b = 0; b < Cfg::kBatch; ++b)
        v[c][b] = s0 + b < ns ? __ldcg(po + static_cast<int64_t>(s0 + b) * D) : 0.f;
    }
  };
  load_batch(0);
  float* wts = wo;         // [G][ns] split weights
  float* lsum = wo + G * ns;  // [G][ns] split sums
  if (warp < G) {
    const float2* ml = p.part_ml + (static_cast<int64_t>(seq) * hq + head0 + warp) * ns;
    float M = -INFINITY;
    for (int s2 = lane; s2 < ns; s2 += 32) {
      const float2 mv2 = __ldcg(ml + s2);
      const float mv = mv2.y > 0.f ? mv2.x : -INFINITY;
      wts[warp * ns + s2] = mv;
      lsum[warp * ns + s2] = mv2.y;
      M = fmaxf(M, mv);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    for (int s2 = lane; s2 < ns; s2 += 32) {
      const float w = M == -INFINITY ? 0.f : ex2(wts[warp * ns + s2] - M);
      wts[warp * ns + s2] = w;
      L = fmaf(w, lsum[warp * ns + s2], L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    __syncwarp();
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int s2 = lane; s2 < ns; s2 += 32) wts[warp * ns + s2] *= inv;
    if (lane == 0) {
      wm[warp] = M;
      wl[warp] = L;
    }
  }
  __syncthreads();
  float out[Cfg::kOut];
#pragma unroll
  for (int c = 0; c < Cfg::kOut; ++c) out[c] = 0.f;
  for (int s0 = 0; s0 < ns; s0 += Cfg::kBatch) {
    if (s0 > 0) load_batch(s0);
#pragma unroll
    for (int c = 0; c < Cfg::kOut; ++c) {
      const int h = (tid + c * kShortThreads) / D;
#pragma unroll
      for (int b = 0; b < Cfg::kBatch; ++b)
        if (s0 + b < ns) out[c] = fmaf(wts[h * ns + s0 + b], v[c][b], out[c]);
    }
  }
#pragma unroll
  for (int c = 0; c < Cfg::kOut; ++c) {
    const int i = tid + c * kShortThreads;
    const int h = i / D, d = i % D;
    p.o[static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
        static_cast<int64_t>(si.q_base) * p.o_stride[1] +
        static_cast<int64_t>(head0 + h) * p.o_stride[2] + d] = __float2bfloat16_rn(out[c]);
    if (d == 0) {
      const float L = wl[h];
      p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
            static_cast<int64_t>(head0 + h) * p.lse_stride[1] + si.q_base] =
          L > 0.f ? (wm[h] + __log2f(L)) * kLn2 : -INFINITY;
    }
  }
  if (tid == 0) *counter = 0;  // ready for the next call on this workspace
}

template <int D, int G>
static int launch_short_dg(const DecodeParams& p, int num_kv_heads, cudaStream_t stream) {
  constexpr int kSmem = ShortCfg<D, G>::kSmemBytes;
  if (kSmem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(decode_short_kernel<D, G>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  const dim3 grid(p.n_split, num_kv_heads, p.layout.batch);
  const cudaError_t e =
      launch_chained(decode_short_kernel<D, G>, grid, dim3(kShortThreads), kSmem, stream, p);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

template <int D>
static int launch_short_d(const DecodeParams& p, int num_kv_heads, cudaStream_t stream) {
  switch (p.group) {
    case 1: return launch_short_dg<D, 1>(p, num_kv_heads, stream);
    case 2: return launch_short_dg<D, 2>(p, num_kv_heads, stream);
    case 3: return launch_short_dg<D, 3>(p, num_kv_heads, stream);
    case 4: return launch_short_dg<D, 4>(p, num_kv_heads, stream);
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
}

int launch_decode_short(int d, const DecodeParams& p, int num_kv_heads, cudaStream_t stream) {
  return d == 256 ? launch_short_d<256>(p, num_kv_heads, stream)
                  : launch_short_d<512>(p, num_kv_heads, stream);
}

}  // namespace g4
