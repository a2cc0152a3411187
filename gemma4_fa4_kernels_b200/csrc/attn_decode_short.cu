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
// CTA (split, KV head, sequence), 256 threads, at most decode_short_keys(D)
// keys (64 for d256, 32 for d512: 32 KB of K and V):
//   1. every K row and V chunk the CTA needs is requested up front (16-B loads
//      into registers), so the whole slice is in flight at once; the group's
//      query vectors go to fp32 shared memory;
//   2. scores: warp w takes keys w, w+8, ...; each lane holds D/32 features of
//      the key row, the group's dot products are reduced across the warp;
//      masked keys get -inf;
//   3. per head the split's max and sum (exp2 domain, as the other kernels);
//   4. O: thread t owns 8 features of one key group (keys g, g+G', ...) and
//      accumulates p * V; the key groups are summed through shared memory.
// One split writes O and LSE directly.  With several splits each CTA writes its
// unnormalised O, max and sum, then takes a ticket on the (sequence, KV head)
// counter; the CTA that takes the last ticket merges every split (exact
// log-sum-exp combination) and resets the counter for the next call.
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

}  // namespace

template <int D, int G>
__global__ void __launch_bounds__(kShortThreads, 2) decode_short_kernel(const DecodeParams p) {
  constexpr int kPerLane = D / 32;               // features of a key row per lane
  constexpr int kLoads = kPerLane / 8;           // 16-B loads per lane and key
  constexpr int kColThreads = D / 8;             // threads covering one V row
  constexpr int kKeyGroups = kShortThreads / kColThreads;
  constexpr int kKeys = decode_short_keys(D);    // keys per CTA at most
  constexpr int kKeysPerWarp = kKeys / kShortWarps;
  constexpr int kKeysPerGroup = kKeys / kKeyGroups;
  __shared__ float qs[G][D];
  __shared__ float ps[G][kKeys];
  __shared__ float red[kKeyGroups][G][D];
  __shared__ float stat[G][2];
  __shared__ int last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const SeqInfo si = p.layout.seq(seq);
  if (si.len_q <= 0) return;  // packed segment without a query token (whole CTA)
  const int q_abs = si.len_k - 1;
  const int k_lo = p.window > 0 ? max(0, q_abs - p.window + 1) : 0;
  const int total = max(0, si.len_k - k_lo);
  const int per = (total + p.n_split - 1) / p.n_split;
  const int kb = k_lo + split * per;
  const int n = min(kKeys, max(0, min(si.len_k, kb + per) - kb));
  const int head0 = kvh * G;

  // Every K row this warp needs is requested before any arithmetic (one or
  // two 16-B loads per lane and key): the loads of a CTA are all in flight at
  // once instead of one latency per key.
  const __nv_bfloat16* kbase = p.k + static_cast<int64_t>(si.b_coord) * p.k_stride[0] +
                               static_cast<int64_t>(kvh) * p.k_stride[2];
  uint4 kraw[kKeysPerWarp][kLoads];
#pragma unroll
  for (int i = 0; i < kKeysPerWarp; ++i) {
    const int j = warp + i * kShortWarps;
    const __nv_bfloat16* row =
        kbase + static_cast<int64_t>(si.k_base + kb + min(j, max(n - 1, 0))) * p.k_stride[1];
#pragma unroll
    for (int l = 0; l < kLoads; ++l)
      kraw[i][l] = j < n ? *reinterpret_cast<const uint4*>(row + l * 256 + lane * 8)
                         : make_uint4(0, 0, 0, 0);
  }
  // and this thread's V rows: K and V of the whole slice are in flight together
  const int vc = tid % kColThreads, vg = tid / kColThreads;
  const __nv_bfloat16* vbase = p.v + static_cast<int64_t>(si.b_coord) * p.v_stride[0] +
                               static_cast<int64_t>(kvh) * p.v_stride[2] + vc * 8;
  uint4 vraw[kKeysPerGroup];
#pragma unroll
  for (int i = 0; i < kKeysPerGroup; ++i) {
    const int j = vg + i * kKeyGroups;
    vraw[i] = j < n ? *reinterpret_cast<const uint4*>(
                          vbase + static_cast<int64_t>(si.k_base + kb + j) * p.v_stride[1])
                    : make_uint4(0, 0, 0, 0);
  }
  for (int i = tid; i < G * D; i += kShortThreads) {
    const int h = i / D, d = i % D;
    qs[h][d] = __bfloat162float(p.q[static_cast<int64_t>(si.b_coord) * p.q_stride[0] +
                                    static_cast<int64_t>(si.q_base) * p.q_stride[1] +
                                    static_cast<int64_t>(head0 + h) * p.q_stride[2] + d]);
  }
  const int qdoc = (p.doc != nullptr && si.len_k > 0) ? p.doc[si.meta_base + q_abs] : 0;
  __syncthreads();

  // ---- scores (log2 domain) ----
  float qr[G][kPerLane];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int l = 0; l < kLoads; ++l)
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[h][l * 8 + e] = qs[h][l * 256 + lane * 8 + e];
#pragma unroll
  for (int i = 0; i < kKeysPerWarp; ++i) {
    const int j = warp + i * kShortWarps;
    float kf[kPerLane];
#pragma unroll
    for (int l = 0; l < kLoads; ++l) bf16x8_to_float(kraw[i][l], kf + l * 8);
    float dot[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < kPerLane; ++e) acc = fmaf(qr[h][e], kf[e], acc);
      dot[h] = acc;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int h = 0; h < G; ++h) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], off);
    if (lane == 0 && j < n) {
      const bool keep = p.doc == nullptr || p.doc[si.meta_base + kb + j] == qdoc;
#pragma unroll
      for (int h = 0; h < G; ++h) ps[h][j] = keep ? dot[h] * kLog2e : -INFINITY;
    }
  }
  __syncthreads();

  // ---- per-head max and sum over this split's keys ----
  if (warp < G) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, ps[warp][j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float msub = m == -INFINITY ? 0.f : m;
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = ex2(ps[warp][j] - msub);  // exp2(-inf) = 0
      ps[warp][j] = e;
      l += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      stat[warp][0] = m;
      stat[warp][1] = l;
    }
  }
  __syncthreads();

  // ---- O = P V over this split's keys ----
  {
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
#pragma unroll
    for (int i = 0; i < kKeysPerGroup; ++i) {
      const int j = vg + i * kKeyGroups;
      if (j < n) {
        float vf[8];
        bf16x8_to_float(vraw[i], vf);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float w = ps[h][j];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[h][e] = fmaf(w, vf[e], acc[h][e]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) red[vg][h][vc * 8 + e] = acc[h][e];
  }
  __syncthreads();

  const int hq = p.num_q_heads;
  if (p.n_split == 1) {
    for (int i = tid; i < G * D; i += kShortThreads) {
      const int h = i / D, d = i % D;
      float o = 0.f;
#pragma unroll
      for (int g = 0; g < kKeyGroups; ++g) o += red[g][h][d];
      const float l = stat[h][1];
      p.o[static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
          static_cast<int64_t>(si.q_base) * p.o_stride[1] +
          static_cast<int64_t>(head0 + h) * p.o_stride[2] + d] =
          __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
      if (d == 0)
        p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
              static_cast<int64_t>(head0 + h) * p.lse_stride[1] + si.q_base] =
            l > 0.f ? (stat[h][0] + __log2f(l)) * kLn2 : -INFINITY;
    }
    return;
  }

  // ---- several splits: partials, then the last arriving CTA merges ----
  const int ns = p.n_split;
  for (int i = tid; i < G * D; i += kShortThreads) {
    const int h = i / D, d = i % D;
    float o = 0.f;
#pragma unroll
    for (int g = 0; g < kKeyGroups; ++g) o += red[g][h][d];
    const int64_t row = (static_cast<int64_t>(seq) * hq + head0 + h) * ns + split;
    p.part_o[row * D + d] = o;
    if (d == 0) p.part_ml[row] = make_float2(stat[h][0], stat[h][1]);
  }
  __threadfence();
  __syncthreads();
  int* counter = p.counters + static_cast<int64_t>(seq) * gridDim.y + kvh;
  if (tid == 0) last = atomicAdd(counter, 1) == ns - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Merge, latency-bound on L2: every split's (max, sum) is fetched in
  // parallel into shared memory (the O reduction buffer, free again), each
  // head's weights 2^(m_s - M) / L are formed once, then every thread sums its
  // features over the splits with independent loads.
  float* wts = &red[0][0][0];                  // [G][ns] weights
  float* sums = wts + G * ns;                  // [G][ns] row sums, then unused
  for (int i = tid; i < G * ns; i += kShortThreads) {
    const int h = i / ns, s2 = i % ns;
    const float2 ml = __ldcg(p.part_ml + (static_cast<int64_t>(seq) * hq + head0 + h) * ns + s2);
    wts[i] = ml.y > 0.f ? ml.x : -INFINITY;
    sums[i] = ml.y;
  }
  __syncthreads();
  if (warp < G) {
    float M = -INFINITY;
    for (int s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, wts[warp * ns + s2]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    for (int s2 = lane; s2 < ns; s2 += 32) {
      const float w = M == -INFINITY ? 0.f : ex2(wts[warp * ns + s2] - M);
      wts[warp * ns + s2] = w;
      L = fmaf(w, sums[warp * ns + s2], L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    __syncwarp();
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int s2 = lane; s2 < ns; s2 += 32) wts[warp * ns + s2] *= inv;
    if (lane == 0) {
      stat[warp][0] = M;
      stat[warp][1] = L;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kShortThreads) {
    const int h = i / D, d = i % D;
    const float* po = p.part_o + (static_cast<int64_t>(seq) * hq + head0 + h) * ns * D + d;
    const float* w = wts + h * ns;
    float acc = 0.f;
#pragma unroll 8
    for (int s2 = 0; s2 < ns; ++s2) acc = fmaf(w[s2], __ldcg(po + static_cast<int64_t>(s2) * D), acc);
    p.o[static_cast<int64_t>(si.b_coord) * p.o_stride[0] +
        static_cast<int64_t>(si.q_base) * p.o_stride[1] +
        static_cast<int64_t>(head0 + h) * p.o_stride[2] + d] = __float2bfloat16_rn(acc);
    if (d == 0) {
      const float L = stat[h][1];
      p.lse[static_cast<int64_t>(si.b_coord) * p.lse_stride[0] +
            static_cast<int64_t>(head0 + h) * p.lse_stride[1] + si.q_base] =
          L > 0.f ? (stat[h][0] + __log2f(L)) * kLn2 : -INFINITY;
    }
  }
  if (tid == 0) *counter = 0;  // ready for the next call on this workspace
}

template <int D>
static int launch_short_d(const DecodeParams& p, int num_kv_heads, cudaStream_t stream) {
  const dim3 grid(p.n_split, num_kv_heads, p.layout.batch);
  switch (p.group) {
    case 1: decode_short_kernel<D, 1><<<grid, kShortThreads, 0, stream>>>(p); break;
    case 2: decode_short_kernel<D, 2><<<grid, kShortThreads, 0, stream>>>(p); break;
    case 3: decode_short_kernel<D, 3><<<grid, kShortThreads, 0, stream>>>(p); break;
    case 4: decode_short_kernel<D, 4><<<grid, kShortThreads, 0, stream>>>(p); break;
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_decode_short(int d, const DecodeParams& p, int num_kv_heads, cudaStream_t stream) {
  return d == 256 ? launch_short_d<256>(p, num_kv_heads, stream)
                  : launch_short_d<512>(p, num_kv_heads, stream);
}

}  // namespace g4
