// Dense Gemma-4 mask builder (g4_build_mask), bit-exact with the reference's
// gemma4_attention_mask (src/gemma4_fa4/masks.py:8-80): a grid-stride loop
// with one thread per (batch, query row, key) element.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gemma4_b200.h"

namespace {

__global__ void build_mask_kernel(uint8_t* __restrict__ out, int batch, int q_len, int kv_len,
                                  int q_off, int window, int bidir, const int* __restrict__ vis,
                                  const int* __restrict__ doc, const uint8_t* __restrict__ pad) {
  const int64_t total = int64_t(batch) * q_len * kv_len;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % kv_len);
    const int64_t bq = i / kv_len;
    const int q = static_cast<int>(bq % q_len) + q_off;
    const int b = static_cast<int>(bq / q_len);
    const int64_t mb = int64_t(b) * kv_len;
    bool allowed = k <= q;
    if (vis && bidir) {
      const int qv = vis[mb + q];
      allowed = allowed || (qv >= 0 && qv == vis[mb + k]);
    }
    if (window > 0) allowed = allowed && (k > q - window);
    if (doc) allowed = allowed && (doc[mb + q] == doc[mb + k]);
    if (pad) allowed = allowed && (pad[mb + k] != 0);
    out[i] = allowed ? 1 : 0;
  }
}

}  // namespace

extern "C" int g4_build_mask(uint8_t* out, int32_t batch, int32_t q_len, int32_t kv_len,
                             int32_t q_start, int32_t window, int32_t allow_vision_bidirectional,
                             const int32_t* vision_ids, const int32_t* document_ids,
                             const uint8_t* key_padding, void* stream) {
  if (batch < 1 || q_len < 0 || kv_len < 0 || window < 0) return G4_ERR_INVALID;
  if (q_start < 0) {
    if (q_len > kv_len) return G4_ERR_INVALID;
    q_start = kv_len - q_len;
  }
  if (int64_t(q_start) + q_len > kv_len) return G4_ERR_INVALID;
  const int64_t total = int64_t(batch) * q_len * kv_len;
  if (total == 0) return G4_OK;
  if (!out) return G4_ERR_INVALID;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int blocks = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
  build_mask_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      out, batch, q_len, kv_len, q_start, window, allow_vision_bidirectional, vision_ids,
      document_ids, key_padding);
  return cudaGetLastError() == cudaSuccess ? G4_OK : G4_ERR_CUDA;
}
