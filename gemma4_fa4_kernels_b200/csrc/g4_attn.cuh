// Problem description shared by the Gemma-4 attention kernels: sequence
// addressing (fixed BSHD or packed THD with cu_seqlens), the exact Gemma mask
// predicate, and the per-Q-tile key-tile range.
//
// Mask (reference masks.py:8-80, h100_masks.py:27-152), with q_abs the query's
// absolute position in its K stream (lower-right alignment, q_abs = q + Sk - Sq,
// plus an optional non-negative causal shift for global layers that ring
// context parallelism uses for blocks of keys that lie wholly before the
// queries; the reference contract has shift 0):
//   window == 0 (global layer):  k <= q_abs
//   window  > 0 (local layer) :  k > q_abs - W
//                                AND (k <= q_abs OR (vis[q_abs] >= 0 AND vis[k] == vis[q_abs]))
//                                AND doc[k] == doc[q_abs]
// where vis defaults to -1 and doc to 0 when the metadata arrays are absent.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace g4 {

constexpr int kTileM = 128;  // query rows per CTA tile
constexpr int kTileN = 128;  // key rows per key tile

struct SeqInfo {
  int seq;      // batch index (fixed) or segment index (packed)
  int b_coord;  // TMA batch coordinate (fixed: seq, packed: 0)
  int q_base;   // first Q token of this sequence along the token axis
  int k_base;   // first K token of this sequence along the token axis
  int len_q;
  int len_k;
  int q_off;          // q_abs - q: len_k - len_q + causal shift
  int64_t meta_base;  // index of key 0 of this sequence in the metadata arrays
};

struct SeqLayout {
  int batch;       // fixed: B; packed: number of segments
  int seqlen_q;    // fixed: Sq; packed: total Tq
  int seqlen_k;    // fixed: Sk; packed: total Tk
  const int* cu_q; // packed only
  const int* cu_k; // packed only
  int64_t meta_stride;  // fixed: per-batch stride of vis/doc; packed: unused
  int causal_shift;     // added to every query's absolute position (global layers)

  __device__ __forceinline__ bool packed() const { return cu_q != nullptr; }

  __device__ __forceinline__ SeqInfo seq(int s) const {
    SeqInfo si;
    si.seq = s;
    if (packed()) {
      si.b_coord = 0;
      si.q_base = cu_q[s];
      si.k_base = cu_k[s];
      si.len_q = cu_q[s + 1] - si.q_base;
      si.len_k = cu_k[s + 1] - si.k_base;
      si.meta_base = si.k_base;
    } else {
      si.b_coord = s;
      si.q_base = 0;
      si.k_base = 0;
      si.len_q = seqlen_q;
      si.len_k = seqlen_k;
      si.meta_base = static_cast<int64_t>(s) * meta_stride;
    }
    si.q_off = si.len_k - si.len_q + causal_shift;
    return si;
  }
};

struct MaskSpec {
  int window;                // 0 = global causal
  const int* vis;            // nullable
  const int* doc;            // nullable
  const int* pair_last;      // nullable: last key with the same (doc, vis) pair (sequence-local)
  const int* pair_first;     // nullable: first position with the same pair (backward only)

  __device__ __forceinline__ bool has_meta() const { return vis != nullptr || doc != nullptr; }
};

// Exact predicate for one (query, key) pair, metadata already fetched.
__device__ __forceinline__ bool mask_allows(int window, int q_abs, int k, int qvis, int qdoc,
                                            int kvis, int kdoc) {
  const bool causal = k <= q_abs;
  if (window == 0) return causal;
  if (k <= q_abs - window) return false;
  if (qdoc != kdoc) return false;
  return causal || (qvis >= 0 && qvis == kvis);
}

// Tile class of key tile [k0, k0+kTileN) for query rows with absolute
// positions [qa0, qa1] when no metadata is present: 0 = skip, 1 = full, 2 = partial.
__device__ __forceinline__ int text_tile_class(int window, int qa0, int qa1, int k0, int len_k) {
  const int k1 = min(k0 + kTileN, len_k) - 1;
  if (k0 > qa1) return 0;
  if (window > 0 && k1 <= qa0 - window) return 0;
  const bool causal_full = (k1 <= qa0) && (k0 + kTileN <= len_k);
  const bool window_full = window == 0 || (k0 > qa1 - window);
  return (causal_full && window_full) ? 1 : 2;
}

}  // namespace g4
