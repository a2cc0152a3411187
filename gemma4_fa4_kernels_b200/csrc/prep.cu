// Fused Gemma-4 Q/K/V preparation: RMS norm (optional learned scale) and
// rotate-half RoPE on the leading rotary_dim features, with the optional
// unscaled, unrotated norm of the same source as a second output, and the
// exact adjoint of both.
//
//   rot   = RoPE(x * r * w)        r = (mean(x^2) + eps)^-1/2
//   plain = x * r
//
// This is the preparation of the reference project's layers: Q = RoPE(QNorm(q)),
// K = RoPE(KNorm(k)), V = VNorm(v) (src/gemma4_fa4/h100_torch_ops.py:302-326,
// :396-403, :456-461) and the global shared-source form K = partial_RoPE(KNorm(Z)),
// V = VNorm(Z) (src/gemma4_fa4/reference.py:306-328).  The backward returns dx
// after both adjoints and the gradient of the learned scale
// (docs/design.md:202-213: dK + dV is not the source gradient).
//
// HBM-bound elementwise work.  A row (one token of one head) is handled by a
// group of LPR = D/16 lanes, two 8-feature chunks per lane (features
// 8(c*LPR + l) .. +8 for chunk c of group lane l), so a warp covers one d512
// row or two d256 rows per step and every lane does the same work for both
// head dims.  Each warp owns a contiguous block of rows (head-fastest, so a
// token's heads arrive back to back and its rotary tables are fetched once),
// keeps a ring of upcoming input rows in shared memory filled by cp.async
// (lane-private slots: each lane reads back only what it copied), exchanges
// rotation partners in registers (the lane's other chunk, or a shuffle
// inside the group), and does the FP32 arithmetic with the packed two-wide
// FP32 instructions.  Outputs are rounded to bf16 once.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_kernels.h"
#include "g4_sm100.cuh"

namespace g4 {
namespace {

constexpr int kPrepWarps = 8;
constexpr int kFwdStages = 4;  // forward: 1 KB of x per stage -> 3 KB in flight per warp
constexpr int kBwdStages = 3;  // backward: x, drot, dplain -> up to 6 KB in flight per warp
constexpr int kStageBytes = 1024;  // one tensor's rows of one warp step (D * 2 * 32 / LPR)
constexpr uint32_t kBf16One2 = 0x3F803F80u;  // two bf16 ones

struct RowAddr {
  int64_t b, s, h;
};

// n / d for n < 2^31 by multiply-high and shift (magic from prep_fastdiv).
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (__umulhi(n, f.mul) + n) >> f.shift;
}

__device__ __forceinline__ RowAddr row_addr(uint32_t row, const PrepParams& p) {
  RowAddr a;
  const uint32_t t = fdiv(row, p.div_heads);
  a.h = row - t * static_cast<uint32_t>(p.heads);
  const uint32_t b = fdiv(t, p.div_seqlen);
  a.s = t - b * static_cast<uint32_t>(p.seqlen);
  a.b = b;
  return a;
}

__device__ __forceinline__ int64_t off3(const int64_t* st, const RowAddr& a) {
  return a.b * st[0] + a.s * st[1] + a.h * st[2];
}

// A chunk is 8 features held as 4 float2 pairs; arithmetic on pairs uses the
// sm_100 packed FP32 instructions (two IEEE operations per instruction).
struct Chunk {
  float2 v[4];
};

__device__ __forceinline__ Chunk unpack8(const uint4& u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  Chunk c;
#pragma unroll
  for (int i = 0; i < 4; ++i) c.v[i] = __bfloat1622float2(h[i]);
  return c;
}

__device__ __forceinline__ uint4 pack8(const Chunk& c) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __float22bfloat162_rn(c.v[i]);
  return u;
}

// Sum over the LPR lanes of a row group (fixed butterfly order).
template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 16-byte global -> shared copy completing asynchronously (L1 bypassed);
// each lane waits for its own copies with cp.async.wait_group.
__device__ __forceinline__ void cp16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Rotation partner values.  rotary_dim R is a power of two; with h8 = R/16
// chunks per half, chunk ci pairs with ci ^ h8.  h8 == LPR pairs the lane's
// two chunks; h8 < LPR pairs chunk 0 of lane l with chunk 0 of lane l ^ h8
// (same group).  Callers use the result only for chunks below R.
template <int LPR>
__device__ __forceinline__ void partner(const Chunk (&x)[2], Chunk (&xp)[2], int h8) {
  if (h8 == LPR) {
    xp[0] = x[1];
    xp[1] = x[0];
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xp[0].v[i].x = __shfl_xor_sync(0xffffffffu, x[0].v[i].x, h8);
    xp[0].v[i].y = __shfl_xor_sync(0xffffffffu, x[0].v[i].y, h8);
  }
}

// The contiguous block of rows of this warp: rows split evenly over the warps
// of the grid (rounded to whole warp steps of 32/LPR rows).
template <int LPR>
__device__ __forceinline__ void warp_rows(uint32_t rows, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t kRpw = 32 / LPR;
  const uint64_t steps = (static_cast<uint64_t>(rows) + kRpw - 1) / kRpw;
  const uint64_t nw = static_cast<uint64_t>(gridDim.x) * kPrepWarps;
  const uint64_t wg = static_cast<uint64_t>(blockIdx.x) * kPrepWarps + (threadIdx.x >> 5);
  lo = static_cast<uint32_t>(steps * wg / nw * kRpw);
  hi = static_cast<uint32_t>(steps * (wg + 1) / nw * kRpw);
  if (hi > rows) hi = rows;
  if (lo > rows) lo = rows;
}

// cos/sin of the lane's rotary chunks for its row's token, kept packed.  On a
// token change the new token's chunks are loaded (normally L1 hits) and the
// next token's lines are prefetched into L1, a whole token's rows ahead.
template <int LPR>
struct Tables {
  uint4 cs[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  uint4 sn[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  int64_t b = -1, s = -1;
  __device__ __forceinline__ void update(const RowAddr& a, const PrepParams& p, int gl, int h8) {
    if (a.b == b && a.s == s) return;
    b = a.b;
    s = a.s;
    const int64_t off = b * p.cs_stride[0] + s * p.cs_stride[1];
    int64_t nb = b, ns = s + 1;
    if (ns == p.seqlen) {
      ns = 0;
      ++nb;
    }
    const bool has_next = nb < p.batch;
    const int64_t noff = nb * p.cs_stride[0] + ns * p.cs_stride[1];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int ci = c * LPR + gl;
      if (ci < 2 * h8) {
        cs[c] = __ldg(reinterpret_cast<const uint4*>(p.cos + off + ci * 8));
        sn[c] = __ldg(reinterpret_cast<const uint4*>(p.sin + off + ci * 8));
        if (has_next) {
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.cos + noff + ci * 8));
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.sin + noff + ci * 8));
        }
      }
    }
  }
};

// Copies one tensor's row (this lane's two chunks) into its ring slots.
template <int LPR>
__device__ __forceinline__ void copy_row(uint4* slot, const __nv_bfloat16* src, int gl) {
#pragma unroll
  for (int c = 0; c < 2; ++c) cp16(slot + c * 32, src + (c * LPR + gl) * 8);
}

template <int LPR>
__global__ void __launch_bounds__(kPrepWarps * 32, 2) prep_fwd_kernel(const PrepParams p) {
  constexpr int D = LPR * 16;
  constexpr int kRpw = 32 / LPR;
  constexpr int kStageU4 = kStageBytes / 16;
  extern __shared__ __align__(16) uint4 prep_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, gl = lane % LPR;  // row within the warp step, lane within the row
  // ring slots of this lane: [stage][chunk][lane] (16-byte units, lane-private)
  uint4* ring = prep_smem + warp * kFwdStages * kStageU4 + lane;
  const int R = p.rotary_dim, h8 = R >> 4;
  uint4 wu[2];  // learned scale, packed bf16
#pragma unroll
  for (int c = 0; c < 2; ++c)
    wu[c] = p.w != nullptr ? *reinterpret_cast<const uint4*>(p.w + (c * LPR + gl) * 8)
                           : make_uint4(kBf16One2, kBf16One2, kBf16One2, kBf16One2);
  uint32_t lo, hi;
  warp_rows<LPR>(p.rows, lo, hi);
  auto issue = [&](uint32_t k) {
    const uint32_t row = lo + k * kRpw + sub;
    if (row < hi)
      copy_row<LPR>(ring + (k % kFwdStages) * kStageU4, p.x + off3(p.x_stride, row_addr(row, p)),
                    gl);
    cp_commit();
  };
#pragma unroll
  for (int k = 0; k < kFwdStages - 1; ++k) issue(k);
  const float inv_d = 1.f / static_cast<float>(D);
  Tables<LPR> tab;
  for (uint32_t k = 0, base = lo; base < hi; ++k, base += kRpw) {
    issue(k + kFwdStages - 1);
    const uint32_t row = base + sub;
    const bool valid = row < hi;
    const RowAddr a = row_addr(valid ? row : base, p);
    if (R > 0 && valid) tab.update(a, p, gl, h8);
    cp_wait<kFwdStages - 1>();
    const uint4* st = ring + (k % kFwdStages) * kStageU4;
    Chunk v[2];
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      v[c] = unpack8(valid ? st[c * 32] : make_uint4(0, 0, 0, 0));
#pragma unroll
      for (int i = 0; i < 4; ++i) acc = __ffma2_rn(v[c].v[i], v[c].v[i], acc);
    }
    const float r = rsqrtf(fmaf(group_sum<LPR>(acc.x + acc.y), inv_d, p.eps));
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[c].v[i] = __fmul2_rn(v[c].v[i], r2);
    if (p.plain != nullptr && valid) {
      __nv_bfloat16* dst = p.plain + off3(p.plain_stride, a) + gl * 8;
#pragma unroll
      for (int c = 0; c < 2; ++c) *reinterpret_cast<uint4*>(dst + c * LPR * 8) = pack8(v[c]);
    }
    if (p.rot == nullptr) continue;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const Chunk w = unpack8(wu[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[c].v[i] = __fmul2_rn(v[c].v[i], w.v[i]);
    }
    if (R > 0) {
      Chunk vp[2];
      partner<LPR>(v, vp, h8);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ci = c * LPR + gl;
        if (ci < 2 * h8) {
          // rot_i = n_i cos_i - n_{i+h} sin_i (i < h), n_i cos_i + n_{i-h} sin_i above
          const Chunk cs = unpack8(tab.cs[c]);
          const Chunk sn = unpack8(tab.sn[c]);
          const float sg = ci < h8 ? -1.f : 1.f;
          const float2 sg2 = make_float2(sg, sg);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 t = __fmul2_rn(__fmul2_rn(vp[c].v[i], sg2), sn.v[i]);
            v[c].v[i] = __ffma2_rn(v[c].v[i], cs.v[i], t);
          }
        }
      }
    }
    if (valid) {
      __nv_bfloat16* dst = p.rot + off3(p.rot_stride, a) + gl * 8;
#pragma unroll
      for (int c = 0; c < 2; ++c) *reinterpret_cast<uint4*>(dst + c * LPR * 8) = pack8(v[c]);
    }
  }
  cp_wait<0>();
}

// Backward.  Ring stages hold the row's x, drot and dplain.  The RoPE adjoint
// partner term g_p * sin_p is formed by the lane owning feature p and
// exchanged like the forward's partner values.
template <int LPR>
__global__ void __launch_bounds__(kPrepWarps * 32, 2) prep_bwd_kernel(const PrepParams p) {
  constexpr int D = LPR * 16;
  constexpr int kRpw = 32 / LPR;
  constexpr int kTensorU4 = kStageBytes / 16;
  constexpr int kStageU4 = 3 * kTensorU4;  // x, drot, dplain
  extern __shared__ __align__(16) uint4 prep_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, gl = lane % LPR;
  uint4* ring = prep_smem + warp * kBwdStages * kStageU4 + lane;
  const int R = p.rotary_dim, h8 = R >> 4;
  const bool has_rot = p.drot != nullptr;
  const bool has_plain = p.dplain != nullptr;
  const bool want_dw = has_rot && p.w != nullptr && p.dw_part != nullptr;
  uint4 wu[2];  // learned scale, packed bf16
  Chunk dw[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) dw[c].v[i] = make_float2(0.f, 0.f);
    wu[c] = p.w != nullptr ? *reinterpret_cast<const uint4*>(p.w + (c * LPR + gl) * 8)
                           : make_uint4(kBf16One2, kBf16One2, kBf16One2, kBf16One2);
  }
  uint32_t lo, hi;
  warp_rows<LPR>(p.rows, lo, hi);
  auto issue = [&](uint32_t k) {
    const uint32_t row = lo + k * kRpw + sub;
    if (row < hi) {
      const RowAddr a = row_addr(row, p);
      uint4* slot = ring + (k % kBwdStages) * kStageU4;
      copy_row<LPR>(slot, p.x + off3(p.x_stride, a), gl);
      if (has_rot) copy_row<LPR>(slot + kTensorU4, p.drot + off3(p.drot_stride, a), gl);
      if (has_plain) copy_row<LPR>(slot + 2 * kTensorU4, p.dplain + off3(p.dplain_stride, a), gl);
    }
    cp_commit();
  };
#pragma unroll
  for (int k = 0; k < kBwdStages - 1; ++k) issue(k);
  const float inv_d = 1.f / static_cast<float>(D);
  Tables<LPR> tab;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (uint32_t k = 0, base = lo; base < hi; ++k, base += kRpw) {
    issue(k + kBwdStages - 1);
    const uint32_t row = base + sub;
    const bool valid = row < hi;
    const RowAddr a = row_addr(valid ? row : base, p);
    if (R > 0 && has_rot && valid) tab.update(a, p, gl, h8);
    cp_wait<kBwdStages - 1>();
    const uint4* st = ring + (k % kBwdStages) * kStageU4;
    Chunk y[2], dy[2];
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      y[c] = unpack8(valid ? st[c * 32] : zero);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc = __ffma2_rn(y[c].v[i], y[c].v[i], acc);
        dy[c].v[i] = make_float2(0.f, 0.f);
      }
    }
    const float r = rsqrtf(fmaf(group_sum<LPR>(acc.x + acc.y), inv_d, p.eps));
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) y[c].v[i] = __fmul2_rn(y[c].v[i], r2);
    if (has_rot) {
#pragma unroll
      for (int c = 0; c < 2; ++c) dy[c] = unpack8(valid ? st[kTensorU4 + c * 32] : zero);
      if (R > 0) {
        // RoPE^T: dn_i = g_i cos_i + g_{i+h} sin_{i+h} (i < h), g_i cos_i - g_{i-h} sin_{i-h}
        Chunk t[2], tp[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int ci = c * LPR + gl;
          if (ci < 2 * h8) {
            const Chunk sn = unpack8(tab.sn[c]);
#pragma unroll
            for (int i = 0; i < 4; ++i) t[c].v[i] = __fmul2_rn(dy[c].v[i], sn.v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) t[c].v[i] = make_float2(0.f, 0.f);
          }
        }
        partner<LPR>(t, tp, h8);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int ci = c * LPR + gl;
          if (ci < 2 * h8) {
            const Chunk cs = unpack8(tab.cs[c]);
            const float sg = ci < h8 ? 1.f : -1.f;
            const float2 sg2 = make_float2(sg, sg);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dy[c].v[i] = __ffma2_rn(dy[c].v[i], cs.v[i], __fmul2_rn(tp[c].v[i], sg2));
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const Chunk w = unpack8(wu[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (want_dw && valid) dw[c].v[i] = __ffma2_rn(dy[c].v[i], y[c].v[i], dw[c].v[i]);
          dy[c].v[i] = __fmul2_rn(dy[c].v[i], w.v[i]);
        }
      }
    }
    if (has_plain) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const Chunk g = unpack8(valid ? st[2 * kTensorU4 + c * 32] : zero);
#pragma unroll
        for (int i = 0; i < 4; ++i) dy[c].v[i] = __fadd2_rn(dy[c].v[i], g.v[i]);
      }
    }
    float2 dot = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) dot = __ffma2_rn(dy[c].v[i], y[c].v[i], dot);
    const float m = group_sum<LPR>(dot.x + dot.y) * inv_d;
    const float2 nm2 = make_float2(-m, -m);
    if (valid) {
      __nv_bfloat16* dst = p.dx + off3(p.dx_stride, a) + gl * 8;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        Chunk o;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o.v[i] = __fmul2_rn(r2, __ffma2_rn(y[c].v[i], nm2, dy[c].v[i]));
        *reinterpret_cast<uint4*>(dst + c * LPR * 8) = pack8(o);
      }
    }
  }
  cp_wait<0>();
  if (!want_dw) return;
  // Per-CTA partial of the scale gradient: the row groups' sums (8 warps x
  // 32/LPR groups) added in a fixed order.
  __syncthreads();
  float* red = reinterpret_cast<float*>(prep_smem);
  const int grp = warp * kRpw + sub;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    float2* dst = reinterpret_cast<float2*>(red + grp * D + (c * LPR + gl) * 8);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = dw[c].v[i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < D; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < kPrepWarps * kRpw; ++g) s += red[g * D + e];
    p.dw_part[static_cast<int64_t>(blockIdx.x) * D + e] = s;
  }
}

// dw[e] = sum over the CTA partials: one warp per feature, lane j summing
// partials j, j + 32, ... in order, then a fixed shuffle tree (deterministic).
__global__ void __launch_bounds__(128) prep_dw_reduce_kernel(const float* part, int n_parts, int d,
                                                             float* dw) {
  const int e = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= d) return;
  float s0 = 0.f, s1 = 0.f;
  int k = lane;
  for (; k + 32 < n_parts; k += 64) {
    s0 += part[static_cast<int64_t>(k) * d + e];
    s1 += part[static_cast<int64_t>(k + 32) * d + e];
  }
  if (k < n_parts) s0 += part[static_cast<int64_t>(k) * d + e];
  float s = s0 + s1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) dw[e] = s;
}

int smem_bytes(bool backward) {
  return backward ? kPrepWarps * kBwdStages * 3 * kStageBytes : kPrepWarps * kFwdStages * kStageBytes;
}

template <typename K>
int grid_for(K kernel, int smem, const PrepParams& p, int sm_count) {
  static_assert(kPrepWarps * 2 * 256 * 4 <= kPrepWarps * kBwdStages * 3 * kStageBytes,
                "the backward ring must hold the dweight reduction rows");
  if (smem > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kPrepWarps * 32, smem) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t rows_per_cta = kPrepWarps * (p.head_dim == 256 ? 2 : 1);
  const int64_t need = (static_cast<int64_t>(p.rows) + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = static_cast<int64_t>(per_sm) * sm_count;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace

FastDiv prep_fastdiv(uint32_t d) {
  FastDiv f{};
  uint32_t s = 0;
  while ((uint64_t{1} << s) < d) ++s;
  f.mul = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << s) - d)) / d + 1);
  f.shift = s;
  return f;
}

int prep_grid(bool backward, const PrepParams& p, int sm_count) {
  const int smem = smem_bytes(backward);
  if (p.head_dim == 256)
    return backward ? grid_for(prep_bwd_kernel<16>, smem, p, sm_count)
                    : grid_for(prep_fwd_kernel<16>, smem, p, sm_count);
  return backward ? grid_for(prep_bwd_kernel<32>, smem, p, sm_count)
                  : grid_for(prep_fwd_kernel<32>, smem, p, sm_count);
}

int launch_prep_fwd(const PrepParams& p, int grid, cudaStream_t stream) {
  const int smem = smem_bytes(false);
  if (p.head_dim == 256)
    prep_fwd_kernel<16><<<grid, kPrepWarps * 32, smem, stream>>>(p);
  else
    prep_fwd_kernel<32><<<grid, kPrepWarps * 32, smem, stream>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int launch_prep_bwd(const PrepParams& p, int grid, cudaStream_t stream) {
  const int smem = smem_bytes(true);
  if (p.head_dim == 256)
    prep_bwd_kernel<16><<<grid, kPrepWarps * 32, smem, stream>>>(p);
  else
    prep_bwd_kernel<32><<<grid, kPrepWarps * 32, smem, stream>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int launch_prep_dw_reduce(const float* part, int n_parts, int d, float* dw, cudaStream_t stream) {
  prep_dw_reduce_kernel<<<(d + 3) / 4, 128, 0, stream>>>(part, n_parts, d, dw);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4
