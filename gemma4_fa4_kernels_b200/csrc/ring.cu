// Ring context parallelism support: merging a block's partial attention into
// a running result, and the fp32 -> bf16 cast of accumulated outputs.
//
// A sequence split across ranks is attended block by block: each block of
// keys gives every query row a partial output O_b (normalised over that block)
// and its log-sum-exp L_b.  Two partials of the same rows combine as
//   L = log(exp(L_a) + exp(L_b)),  O = O_a exp(L_a - L) + O_b exp(L_b - L),
// which is exact: softmax over the union of the key blocks.  A row that no
// block reached keeps L = -inf and O = 0.  The running O stays in fp32.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "g4_kernels.h"

namespace g4 {

// One warp per (token, head): the two LSEs, then the row's D features in
// chunks of eight per lane (fp32 running output, bf16 block output).
__global__ void merge_partial_kernel(const MergeParams p) {
  pdl_enter();
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(p.tokens) * p.heads;
  if (warp >= rows) return;
  const int64_t t = warp / p.heads;
  const int h = static_cast<int>(warp % p.heads);
  float* la_p = p.lse_acc + h * p.lse_acc_stride[0] + t * p.lse_acc_stride[1];
  const float la = *la_p;
  const float lb = p.lse_part[h * p.lse_part_stride[0] + t * p.lse_part_stride[1]];
  const float m = fmaxf(la, lb);
  float wa = 1.f, wb = 0.f, l = la;
  if (m != -INFINITY) {
    const float ea = expf(la - m), eb = expf(lb - m);  // exp(-inf) = 0
    const float s = ea + eb;
    wa = ea / s;
    wb = eb / s;
    l = m + logf(s);
  }
  float* oa = p.o_acc + t * p.o_acc_stride[0] + h * p.o_acc_stride[1];
  const __nv_bfloat16* ob = p.o_part + t * p.o_part_stride[0] + h * p.o_part_stride[1];
  for (int c = lane * 8; c < p.head_dim; c += 256) {
    float4 a0 = *reinterpret_cast<const float4*>(oa + c);
    float4 a1 = *reinterpret_cast<const float4*>(oa + c + 4);
    const uint4 braw = *reinterpret_cast<const uint4*>(ob + c);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&braw);
    const float2 b01 = __bfloat1622float2(b2[0]), b23 = __bfloat1622float2(b2[1]);
    const float2 b45 = __bfloat1622float2(b2[2]), b67 = __bfloat1622float2(b2[3]);
    a0.x = a0.x * wa + b01.x * wb;
    a0.y = a0.y * wa + b01.y * wb;
    a0.z = a0.z * wa + b23.x * wb;
    a0.w = a0.w * wa + b23.y * wb;
    a1.x = a1.x * wa + b45.x * wb;
    a1.y = a1.y * wa + b45.y * wb;
    a1.z = a1.z * wa + b67.x * wb;
    a1.w = a1.w * wa + b67.y * wb;
    *reinterpret_cast<float4*>(oa + c) = a0;
    *reinterpret_cast<float4*>(oa + c + 4) = a1;
  }
  if (lane == 0) *la_p = l;
}

int launch_merge_partial(const MergeParams& p, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.tokens) * p.heads;
  if (rows <= 0) return 0;
  const int64_t blocks = (rows * 32 + 255) / 256;
  cudaError_t e = launch_chained(merge_partial_kernel, dim3(static_cast<unsigned>(blocks)),
                                 dim3(256), 0, stream, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4

namespace g4 {

// dst += src over n floats (n a multiple of 4, both 16-byte aligned): the
// halo key gradients a rank receives back from its successor.
__global__ void add_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n4) {
  pdl_enter();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(dst)[i];
    const float4 b = reinterpret_cast<const float4*>(src)[i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    reinterpret_cast<float4*>(dst)[i] = a;
  }
}

int launch_add_f32(float* dst, const float* src, int64_t n, cudaStream_t stream) {
  const int64_t n4 = n / 4;
  if (n4 <= 0) return 0;
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 148 * 8);
  cudaError_t e = launch_chained(add_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256),
                                 0, stream, dst, src, n4);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4
