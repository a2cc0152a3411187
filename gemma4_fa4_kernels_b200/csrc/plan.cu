// Device-side planning for packed (cu_seqlens) inputs and metadata masks.
//
// * plan_tiles: turns cu_seqlens into a compact (segment, tile) work list so
//   that a fixed-size grid (an upper bound known on the host without reading
//   cu_seqlens) covers every tile of every segment; no host synchronisation.
// * pair_last / pair_first: for every position with a non-negative vision id,
//   the last / first position of the same sequence carrying the same
//   (document, vision) pair.  A query's allowed keys extend rightwards exactly
//   to pair_last (the vision exception has no right window cap, reference
//   masks.py:55-66), which bounds the key tiles a query tile visits; a key is
//   seen by earlier queries down to pair_first, which bounds the query tiles
//   a key tile visits in the backward pass.  The reference builds the equivalent
//   information on the host per segment (sparse_schedule.py:146-178, the
//   pair_blocks index); here one CTA per sequence uses a shared-memory hash
//   table.  If the table overflows, the bound falls back to the sequence end,
//   which is conservative (tiles are still masked element by element).
#include <cuda_runtime.h>
#include <stdint.h>

#include "g4_kernels.h"

namespace g4 {

__global__ void plan_tiles_kernel(const int* __restrict__ cu, int nseg, int tile, int2* tiles,
                                  int* n_tiles, int* seg_first) {
  __shared__ int scan[1024];
  __shared__ int carry;
  pdl_enter();
  const int tid = threadIdx.x;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nseg; base += 1024) {
    const int s = base + tid;
    const int len = s < nseg ? cu[s + 1] - cu[s] : 0;
    const int cnt = len > 0 ? (len + tile - 1) / tile : 0;
    scan[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {  // inclusive Hillis-Steele scan
      const int v = tid >= off ? scan[tid - off] : 0;
      __syncthreads();
      scan[tid] += v;
      __syncthreads();
    }
    const int start = carry + scan[tid] - cnt;
    for (int t = 0; t < cnt; ++t) tiles[start + t] = make_int2(s, t);
    if (seg_first && s < nseg) seg_first[s] = start;
    __syncthreads();
    if (tid == 1023) carry += scan[1023];
    __syncthreads();
  }
  if (tid == 0) *n_tiles = carry;
}

int launch_plan_tiles(const int* cu, int nseg, int tile, int2* tiles, int* n_tiles,
                      int* seg_first, cudaStream_t stream) {
  cudaError_t e = launch_chained(plan_tiles_kernel, dim3(1), dim3(1024), 0, stream, cu, nseg,
                                 tile, tiles, n_tiles, seg_first);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

constexpr int kHashCap = 2048;  // distinct (document, vision) pairs per sequence
constexpr unsigned long long kHashEmpty = ~0ull;

__device__ __forceinline__ unsigned hash_key(unsigned long long key) {
  key ^= key >> 33;
  key *= 0xff51afd7ed558ccdull;
  key ^= key >> 33;
  return static_cast<unsigned>(key) & (kHashCap - 1);
}

__global__ void pair_last_kernel(SeqLayout layout, const int* __restrict__ vis,
                                 const int* __restrict__ doc, int* __restrict__ pair_last,
                                 int* __restrict__ pair_first) {
  __shared__ unsigned long long keys[kHashCap];
  __shared__ int last[kHashCap];
  __shared__ int first[kHashCap];
  __shared__ int overflow;
  const SeqInfo si = layout.seq(blockIdx.x);
  for (int i = threadIdx.x; i < kHashCap; i += blockDim.x) {
    keys[i] = kHashEmpty;
    last[i] = -1;
    first[i] = 0x7fffffff;
  }
  if (threadIdx.x == 0) overflow = 0;
  __syncthreads();
  // vis >= 0, so the packed key never equals the all-ones empty marker.
  for (int k = threadIdx.x; k < si.len_k; k += blockDim.x) {
    const int v = vis[si.meta_base + k];
    if (v < 0) continue;
    const int d = doc ? doc[si.meta_base + k] : 0;
    const unsigned long long key =
        (static_cast<unsigned long long>(static_cast<unsigned>(d)) << 32) | static_cast<unsigned>(v);
    unsigned h = hash_key(key);
    bool placed = false;
    for (int probe = 0; probe < kHashCap; ++probe) {
      const unsigned long long prev = atomicCAS(&keys[h], kHashEmpty, key);
      if (prev == kHashEmpty || prev == key) {
        atomicMax(&last[h], k);
        atomicMin(&first[h], k);
        placed = true;
        break;
      }
      h = (h + 1) & (kHashCap - 1);
    }
    if (!placed) overflow = 1;
  }
  __syncthreads();
  for (int k = threadIdx.x; k < si.len_k; k += blockDim.x) {
    const int v = vis[si.meta_base + k];
    int out = k, out_first = k;
    if (v >= 0) {
      if (overflow) {
        out = si.len_k - 1;
        out_first = 0;
      } else {
        const int d = doc ? doc[si.meta_base + k] : 0;
        const unsigned long long key =
            (static_cast<unsigned long long>(static_cast<unsigned>(d)) << 32) |
            static_cast<unsigned>(v);
        unsigned h = hash_key(key);
        for (int probe = 0; probe < kHashCap; ++probe) {
          if (keys[h] == key) {
            out = max(k, last[h]);
            out_first = min(k, first[h]);
            break;
          }
          h = (h + 1) & (kHashCap - 1);
        }
      }
    }
    pair_last[si.meta_base + k] = out;
    if (pair_first) pair_first[si.meta_base + k] = out_first;
  }
}

int launch_pair_last(const SeqLayout& layout, const int* vis, const int* doc, int* pair_last,
                     int* pair_first, int nseq, cudaStream_t stream) {
  if (nseq <= 0) return 0;
  pair_last_kernel<<<nseq, 1024, 0, stream>>>(layout, vis, doc, pair_last, pair_first);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace g4
