// Internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "g4_attn.cuh"

namespace g4 {

// Chained launches (programmatic dependent launch).  The attention kernels of
// one call run back to back on a stream; launched with launch_chained, a
// kernel is launched ahead and its CTAs are dispatched as the previous
// kernel's CTAs exit, instead of after a full launch gap.  A kernel launched
// this way calls pdl_enter() before its first access to memory that an earlier
// kernel of the call writes: it waits until the previous grid in the stream has
// completed and its writes are visible (a predecessor that is not a chained
// kernel passes at once).  Most kernels wait at their start; the backward
// preprocess and the range planner of fixed layouts without key-tile lists
// (which touch nothing an earlier kernel of the call writes) wait at their end,
// and the short-window decode before its first arrival counter, so they run
// under their predecessor; every chained kernel waits somewhere, so its
// completion implies its predecessor's.
// The attention kernels give no early trigger (griddepcontrol.launch_dependents):
// with one, the successor's waiting CTAs took SMs during the long c1 kernels'
// last wave and the step got 1% slower; without it c0 is 3% and c1 0.6% faster.
// Only a predecessor whose successor works before it waits triggers at its
// start: the one-CTA workspace reset, and the backward preprocess when the
// late-waiting range planner follows.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
#endif

template <typename... Exp, typename... Act>
inline cudaError_t launch_chained(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// Key-tile list entries written by plan_qtile_lists_kernel: the key tile's
// index in the low 30 bits, kTileEntryFull when every pair of the tile (valid
// rows and keys) is allowed, kTileEntryText when the window / causal range
// rule alone is exact on the tile (no key of the tile is a vision token, and
// every valid row and key of it lie in one document).
constexpr int kTileEntryIndex = 0x3fffffff;
constexpr int kTileEntryText = 0x40000000;
constexpr int kTileEntryFull = static_cast<int>(0x80000000u);

struct FwdParams {
  SeqLayout layout;
  MaskSpec mask;
  int group;                       // query heads per KV head
  __nv_bfloat16* o;
  int64_t o_stride[3];             // batch, token, head (elements)
  float* lse;
  int64_t lse_stride[2];           // batch, head (floats); token stride 1
  const int2* tiles;               // packed: (segment, q tile) work list, else null
  const int* n_tiles;
  // metadata masks: per query tile (flattened index) the exact key-tile list
  // from plan_qtile_lists_kernel (entries tagged as kTileEntry* describes) and
  // its count in ranges[g].y; null for text masks
  const int4* ranges;
  const int* klist;
  int klist_stride;
  int* err;                        // device error word
};

struct BwdParams {
  SeqLayout layout;
  MaskSpec mask;
  int group;
  int num_q_heads;
  const __nv_bfloat16* o;
  int64_t o_stride[3];
  const __nv_bfloat16* dout;
  int64_t do_stride[3];
  const float* lse;                // natural-log LSE from the forward
  int64_t lse_stride[2];
  const float* dlse;               // nullable, same layout as lse
  float* delta;                    // workspace: rowsum(dO*O) - dLSE, [head][token]
  float* lse2;                     // workspace: LSE * log2(e), [head][token]
  int64_t ws_head_stride;          // token count of the workspace rows
  __nv_bfloat16* dq;
  int64_t dq_stride[3];
  __nv_bfloat16* dk;
  int64_t dk_stride[3];
  __nv_bfloat16* dv;
  int64_t dv_stride[3];
  const int2* q_tiles;             // packed: (segment, q tile) work list
  const int* n_q_tiles;
  const int2* k_tiles;             // packed: (segment, k tile) work list
  const int* n_k_tiles;
  int* err;
};

// Backward with materialised P / dS scratch tiles (attn_bwd_mat.cu), and the
// two-pass d512 forward that shares its kernels.
//
// Work is cut into bands: a band is a set of KV heads (with all their query
// heads) and up to two ranges of the flattened query-tile list.  One band's
// P / dS tiles fit the scratch, so any problem size runs the same kernels, one
// launch set per band.  A band that holds every query tile writes dV / dK as
// bf16 like the query-major products; with several query bands the dV / dK
// partial sums of each band are added in fp32 (TMA reduce-add) into a buffer
// that a final kernel converts.
struct MatParams {
  SeqLayout layout;
  MaskSpec mask;                   // window and documents only (no vision)
  int group;
  int num_q_heads;
  int n_qt_fixed;                  // fixed layout: query tiles per sequence
  const int2* q_tiles;             // packed: (segment, q tile) list, else null
  const int* n_q_tiles;
  const int2* k_tiles;
  const int* n_k_tiles;
  const int* seg_first_qtile;      // packed: list index of each segment's first q tile
  int4* ranges;                    // per query tile: kt_lo, n_kt, scratch prefix, sequence
  const int* klist;                // nullable: per query tile its key tiles (metadata masks)
  int klist_stride;                // entries reserved per query tile in klist
  int64_t head_cap_tiles;          // scratch tiles reserved per query head of a band
  // this launch set's band
  int band_g[4];                   // query tiles [band_g[0], band_g[1]) and [band_g[2], band_g[3])
  int band_h0;                     // first KV head
  int band_nh;                     // KV heads
  int kv_item0;                    // key-major grids: first work item (key tile) of the band
  // fp32 accumulation: the product adds into an fp32 tensor (TMA reduce-add;
  // direct atomics for partial tiles of packed segments) instead of storing bf16
  int acc_kv;                      // dV / dK
  int acc_q;                       // dQ
  float* dq_acc;
  int64_t dq_acc_stride[3];
  float* dk_acc;
  int64_t dk_acc_stride[3];
  float* dv_acc;
  int64_t dv_acc_stride[3];
  uint8_t* p_tiles;
  uint8_t* ds_tiles;
  const float* lse2;
  const float* delta;
  int64_t ws_head_stride;
  __nv_bfloat16* dq;
  int64_t dq_stride[3];
  __nv_bfloat16* dk;
  int64_t dk_stride[3];
  __nv_bfloat16* dv;
  int64_t dv_stride[3];
  // two-pass forward (d512): pass 1 writes P (in p_tiles, relative to the
  // running row max), the per-row rescale factor of every tile, a per-tile
  // "some row rescaled" flag, 1/rowsum and the LSE; pass 2 forms O = P V.
  float* fwd_alpha;                // [band head][tile][128]
  int* fwd_flags;                  // [band head][tile]
  float* fwd_inv_l;                // [head][token]
  float* lse_out;
  int64_t lse_stride[2];
  __nv_bfloat16* o;
  int64_t o_stride[3];
  int* err;
};

// Single-token decode against a (static) KV cache (attn_decode.cu): one query
// token per sequence, keys split across CTAs, partial results merged by a
// second kernel unless one split covers the whole key range.
struct DecodeParams {
  SeqLayout layout;                // fixed: Sq == 1; packed: every segment has <= 1 query
  int window;                      // 0 = global
  const int* doc;                  // nullable; local layers only
  int group;                       // query heads per KV head, <= kDecodeMaxGroup
  int num_q_heads;
  int n_split;                     // key-range splits per (sequence, KV head)
  const __nv_bfloat16* q;
  int64_t q_stride[3];             // batch, token, head (elements)
  __nv_bfloat16* o;
  int64_t o_stride[3];
  float* lse;
  int64_t lse_stride[2];           // batch, head (floats); token stride 1
  float* part_o;                   // [seq][Hq][n_split][D] unnormalised O (n_split > 1)
  float2* part_ml;                 // [seq][Hq][n_split] (running max log2, row sum)
  int* err;
  // short-window kernel (attn_decode_short.cu): raw K/V and the per-(sequence,
  // KV head) arrival counters of its fused merge (zero at launch)
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t k_stride[3];
  int64_t v_stride[3];
  int* counters;
};
constexpr int kDecodeMaxGroup = 16;
// Short-window decode: CUDA-core dot products, one launch (the last CTA of a
// (sequence, KV head) merges the splits); query groups of at most 4 heads and
// at most decode_short_keys(D, G) keys per CTA.
constexpr int kDecodeShortMaxGroup = 4;
// the merge holds every split's weight of the group's heads in shared memory
constexpr int kDecodeShortMaxSplits = 1024;
// keys per CTA, held in registers: 32 KB of K and V rows in flight per CTA
// (64 keys at d256, 32 at d512), half that for groups of 3 or 4 heads (whose
// query features take the registers)
__host__ __device__ constexpr int decode_short_keys(int d, int g) {
  return (g > 2 ? 8192 : 16384) / d;
}
int launch_decode_short(int d, const DecodeParams& p, int num_kv_heads, cudaStream_t stream);
constexpr int kDecodeMaxSplits = 1024;
constexpr int kDecodeStages = 6;   // 32 KB ring stages
int decode_smem_bytes(int d);
int launch_decode(int d, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                  int num_kv_heads, cudaStream_t stream);
int launch_decode_combine(int d, const DecodeParams& p, cudaStream_t stream);

// Fused Q/K/V preparation (prep.cu): rows (b, s, h) of head_dim features,
// strides in elements [batch, token, head]; cos/sin (batch, token, rotary_dim)
// with strides [batch, token] (batch stride may be 0).
struct FastDiv {
  uint32_t mul, shift;             // n / d = (umulhi(n, mul) + n) >> shift for n < 2^31
};
FastDiv prep_fastdiv(uint32_t d);
struct PrepParams {
  int batch, seqlen, heads, head_dim, rotary_dim;
  uint32_t rows;                   // batch * seqlen * heads (< 2^31)
  FastDiv div_heads, div_seqlen;
  float eps;
  const __nv_bfloat16* x;
  int64_t x_stride[3];
  const __nv_bfloat16* w;          // nullable learned scale (head_dim)
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t cs_stride[2];
  __nv_bfloat16* rot;              // forward: RoPE(Norm(x) * w), nullable
  int64_t rot_stride[3];
  __nv_bfloat16* plain;            // forward: Norm(x), nullable
  int64_t plain_stride[3];
  const __nv_bfloat16* drot;       // backward cotangents, nullable
  int64_t drot_stride[3];
  const __nv_bfloat16* dplain;
  int64_t dplain_stride[3];
  __nv_bfloat16* dx;
  int64_t dx_stride[3];
  float* dw_part;                  // backward: [grid][head_dim] partials (nullable)
};
int prep_grid(bool backward, const PrepParams& p, int sm_count);
int launch_prep_fwd(const PrepParams& p, int grid, cudaStream_t stream);
int launch_prep_bwd(const PrepParams& p, int grid, cudaStream_t stream);
int launch_prep_dw_reduce(const float* part, int n_parts, int d, float* dw, cudaStream_t stream);
// bounded-wait self-test (one CTA): see g4_selftest_wait
int launch_selftest_wait(int mode, int* err, unsigned long long* out, cudaStream_t stream);

// Ring context parallelism (ring.cu): o_acc / lse_acc <- merge with a block's
// partial (o_part bf16, lse_part); strides in elements, feature stride 1.
struct MergeParams {
  float* o_acc;
  float* lse_acc;
  const __nv_bfloat16* o_part;
  const float* lse_part;
  int64_t o_acc_stride[2];     // token, head
  int64_t o_part_stride[2];
  int64_t lse_acc_stride[2];   // head, token
  int64_t lse_part_stride[2];
  int tokens, heads, head_dim;
};
int launch_merge_partial(const MergeParams& p, cudaStream_t stream);
int launch_add_f32(float* dst, const float* src, int64_t n, cudaStream_t stream);

int launch_plan_qtile_ranges(const MatParams& p, cudaStream_t stream);
// metadata masks: exact key-tile lists per query tile into p.klist (and the
// counts into p.ranges); run before launch_plan_qtile_ranges
int launch_plan_qtile_lists(const MatParams& p, int n_qt_total, cudaStream_t stream);
// fp32 [token][head][d] (contiguous) -> bf16 with strides: the final dV / dK of
// a multi-band backward (or any fp32 gradient accumulator)
int launch_cast_f32_bf16(const float* src, int64_t rows, int heads, int d,
                         __nv_bfloat16* dst, const int64_t* dst_stride, int batch,
                         int64_t rows_per_batch, cudaStream_t stream);
// pass: d512 runs pass 0 (P) then pass 1 (dS); d256 computes both in pass 0;
// pass 2 is the forward's first pass (online softmax, d512 only).
int launch_bwd_score(int d, int pass, const CUtensorMap& tq, const CUtensorMap& tk,
                     const CUtensorMap& tv, const CUtensorMap& tdo, const MatParams& p, int grid_x,
                     cudaStream_t stream);
// which: 0 = dV (B = dO), 1 = dK (B = Q), 2 = dQ (B = K), 3 = forward O = P V
// (B = V); tb uses 64-row boxes, tout (the output: dV, dK, dQ or O) 128-row boxes.
// ta (nullable): the A scratch (dS for dQ, P for O) viewed as bytes, (256, 64,
// half tiles) with (256, 64, 1) boxes; given it, the d512 dQ and O GEMMs run as
// CTA pairs.
int launch_bwd_tile_gemm(int d, int which, const CUtensorMap& tb, const CUtensorMap& tout,
                         const CUtensorMap* ta, const MatParams& p, int grid_x, int grid_y,
                         cudaStream_t stream);
bool gemm_pairs_ok(int d, int which, const MatParams& p);
// dV = P^T dO and dK = dS^T Q in one launch (KV-major CTAs of the two products
// interleaved): tdo / tq with 64-row boxes, tdv / tdk with 128-row boxes.
int launch_bwd_tile_gemm_dvdk(int d, const CUtensorMap& tdo, const CUtensorMap& tdv,
                              const CUtensorMap& tq, const CUtensorMap& tdk, const MatParams& p,
                              int grid_x, int grid_y, cudaStream_t stream);

template <int DQK>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
               const FwdParams& p, int grid_x, int num_q_heads, int slabs, cudaStream_t stream);

// Persistent local forward (d256): `ctas` CTAs walk every (head, query tile) item.
int launch_fwd_persistent(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const FwdParams& p, int ctas, int num_q_heads, cudaStream_t stream);

// early_trigger: the next launch is the range planner of a fixed layout without
// key-tile lists, which waits for the preprocess only at its end.
int launch_bwd_preprocess(const BwdParams& p, int head_dim_v, int64_t tokens_q,
                          bool early_trigger, cudaStream_t stream);

// dQ: grid (grid_x query tiles, Hq, D/256 slabs).  Maps: Q/K/V/dO with 128-row
// boxes and K with 64-row boxes.
template <int D>
int launch_bwd_dq(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tk64,
                  const CUtensorMap& tv, const CUtensorMap& tdo, const BwdParams& p, int grid_x,
                  cudaStream_t stream);

// dK/dV: grid (grid_x key tiles, Hkv, D/128 slabs).  Maps with 128-row boxes.
template <int D>
int launch_bwd_dkv(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const CUtensorMap& tdo, const BwdParams& p, int grid_x, cudaStream_t stream);

// planning kernels (plan.cu)
int launch_plan_tiles(const int* cu, int nseg, int tile, int2* tiles, int* n_tiles,
                      int* seg_first, cudaStream_t stream);
int launch_pair_last(const SeqLayout& layout, const int* vis, const int* doc, int* pair_last,
                     int* pair_first, int nseq, cudaStream_t stream);

}  // namespace g4
