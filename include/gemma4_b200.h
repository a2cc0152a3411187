/*
 * gemma4_b200.h -- C ABI of the B200 (sm_100a) Gemma-4 attention library
 * (libgemma4_b200.so).
 *
 * The reference project reaches its GPU kernels through the FlashAttention-4
 * CuTe-DSL Python interface; these entry points are the native boundary that
 * replaces those calls.  Each declaration names the reference call site it
 * stands in for (paths inside amazingvince/gemma4-fa4-kernels).
 *
 * Conventions
 *  - All tensors are device pointers owned by the caller; the library never
 *    allocates or frees caller memory.  Scratch memory is passed in as
 *    `workspace` (size from the matching *_workspace_bytes query, base
 *    16-byte aligned).
 *  - Q/K/V/O and gradients are bf16 with unit stride along the head dimension;
 *    the other strides are in elements and must be multiples of 8 (16 bytes),
 *    base pointers 16-byte aligned.  LSE/dLSE are fp32 natural-log values.
 *  - Fixed layout (cu_seqlens_q == NULL): Q (B,Sq,Hq,D), K/V (B,Sk,Hkv,D),
 *    LSE (B,Hq,Sq).  Packed layout: Q (Tq,Hq,D), K/V (Tk,Hkv,D), LSE (Hq,Tq),
 *    cu_seqlens int32 (B+1); each query segment is the lower-right suffix of
 *    its key segment.
 *  - softmax scale is exactly 1.0.  window == 0 selects the global causal mask;
 *    window > 0 the local mask  k > q-W AND (k <= q OR same vision id >= 0)
 *    AND same document id (vision/document ids follow the K stream).
 *  - Calls are asynchronous on `stream` (a cudaStream_t, NULL = legacy default)
 *    and return G4_OK or an error code; g4_last_error() describes the last
 *    failure of the calling thread.  All argument checks happen before any
 *    launch.
 */
#ifndef GEMMA4_B200_H_
#define GEMMA4_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_ABI_VERSION 2

enum g4_status {
  G4_OK = 0,
  G4_ERR_INVALID = 1,     /* malformed arguments (reference: ValueError) */
  G4_ERR_UNSUPPORTED = 2, /* outside the supported contract (reference: UnsupportedH100Path) */
  G4_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  G4_ERR_DEVICE = 4,      /* a kernel reported a device-side failure (bounded wait expired) */
  G4_ERR_WORKSPACE = 5    /* workspace missing or too small */
};

typedef struct g4_attn_args {
  /* forward operands */
  const void* q;
  const void* k;
  const void* v;
  void* o;          /* forward output; backward input */
  float* lse;       /* forward output; backward input */
  /* backward operands (ignored by the forward) */
  const void* dout;
  const float* dlse; /* nullable: gradient w.r.t. LSE */
  void* dq;
  void* dk;
  void* dv;
  /* strides in elements: [batch, token, head]; batch ignored for packed */
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t do_stride[3];
  int64_t dq_stride[3];
  int64_t dk_stride[3];
  int64_t dv_stride[3];
  int64_t lse_stride[2]; /* [batch, head] in floats; token stride is 1 */
  /* geometry */
  int32_t batch;        /* fixed: B; packed: number of segments */
  int32_t seqlen_q;     /* fixed: Sq; packed: total Tq */
  int32_t seqlen_k;     /* fixed: Sk; packed: total Tk */
  const int32_t* cu_seqlens_q; /* packed only, device, B+1 entries */
  const int32_t* cu_seqlens_k;
  int32_t max_seqlen_q; /* packed: maxima of the segment lengths */
  int32_t max_seqlen_k;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim_qk;  /* 256 (local) or 512 (global) */
  int32_t head_dim_v;   /* equal to head_dim_qk */
  int32_t window;       /* 0 = global causal; > 0 = sliding window W */
  /* contiguous int32 metadata along the K stream: fixed (B,Sk), packed (Tk,); nullable */
  const int32_t* vision_ids;
  const int32_t* document_ids;
  /* scratch */
  void* workspace;
  size_t workspace_bytes;
  /* ABI 2 */
  int32_t causal_shift;    /* global layers (window == 0) only: added to every query's
                              position, q_abs = q + Sk - Sq + shift, shift >= 0 (the reference
                              contract is 0).  shift >= Sq makes every key visible: ring context
                              parallelism's blocks of keys that precede the queries.  In the
                              fixed layout Sq may exceed Sk by at most the shift. */
  int32_t grad_accumulate; /* backward: 0 = dq/dk/dv are bf16 and overwritten; 1 = they are fp32
                              (strides in fp32 elements, multiples of 8) and the gradients are
                              added to their contents (partial sums over ring steps) */
} g4_attn_args;

/* ABI version of the loaded library (G4_ABI_VERSION). */
int g4_abi_version(void);

/* Description of the last failure on the calling thread ("" if none). */
const char* g4_last_error(void);

/*
 * Workspace bytes for g4_attn_fwd (no device access).  For global d512 the
 * full size lets the forward run in two passes (S and the online softmax
 * once, writing bf16 P tiles to HBM scratch; then O = P V with one 512-column
 * accumulator), avoiding the second QK^T of a split-output kernel; the
 * minimum size runs the single-kernel forward.  g4_attn_fwd picks the
 * two-pass path whenever it is eligible and workspace_bytes is at least the
 * full size.
 */
size_t g4_attn_fwd_workspace_bytes(const g4_attn_args* args);
size_t g4_attn_fwd_min_workspace_bytes(const g4_attn_args* args);

/*
 * Attention forward: O and LSE.
 * Replaces the FA4 forward launches of src/gemma4_fa4/h100.py:
 *   flash_attn_func (fa4_local_text_forward :766-778, fa4_local_forward :800-815,
 *   fa4_global_forward_only :1013-1036, _FA4GlobalTextFunction.forward :1352-1386)
 *   flash_attn_varlen_func (fa4_local_varlen_forward :864-910,
 *   _run_global_varlen_slabs :1174-1190).
 * The global d512 output is produced in one launch, not two V256 slab calls.
 */
int g4_attn_fwd(const g4_attn_args* args, void* stream);

/*
 * Workspace bytes for g4_attn_bwd (no device access).  The full size lets the
 * backward materialise P and dS once as bf16 scratch tiles in HBM (every
 * backward matmul done exactly once; about 64 KB per query head and visible
 * 128x128 tile); the minimum size runs kernels that recompute S and dP
 * instead.  g4_attn_bwd picks the materialised path whenever it is eligible
 * (no vision metadata) and workspace_bytes is at least the full size.
 */
size_t g4_attn_bwd_workspace_bytes(const g4_attn_args* args);
size_t g4_attn_bwd_min_workspace_bytes(const g4_attn_args* args);

/*
 * Attention backward: dQ, dK, dV from (Q, K, V, O, LSE, dO[, dLSE]).
 * Replaces FA4's autograd backward for the local adapters (h100.py:766-910)
 * and flash_attn.cute.interface._flash_attn_bwd_gemma4_global_d512
 * (patches/flash-attention/0002-...patch:1021-1512, called from
 * h100.py:1304-1317 and :1389-1394).  dQ/dK/dV are fully overwritten;
 * keys no query attends to receive exact zeros.
 */
int g4_attn_bwd(const g4_attn_args* args, void* stream);

/*
 * Backward that allocates nothing, for callers that cannot allocate device
 * memory at call time (no reference counterpart: the reference allocates its
 * backward workspaces with torch).  Examples: a runtime that plans all device
 * memory ahead of time and forbids cudaMalloc while it executes, or a plugin
 * host that hands an op its tensors but no scratch buffer.  Same arguments
 * and results as g4_attn_bwd, except that `workspace`/`workspace_bytes` are
 * ignored: scratch comes from one static device array of
 * G4_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads the
 * library keeps until process exit.  The arguments are checked first; then a
 * call whose minimum scratch need (g4_attn_bwd_min_workspace_bytes) exceeds
 * the array fails with G4_ERR_WORKSPACE before any launch.  Within the array
 * the backward takes its fastest form that fits (see g4_attn_bwd).  Every call
 * asks the runtime for the array's address on the current device; the first
 * call on a device also loads the library's kernels there, so make it before
 * any CUDA graph capture.  All calls share the one array and its contents
 * persist between calls: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller.  A bounded wait that
 * expired inside such a call is read back with
 * g4_attn_bwd_noalloc_device_error.
 */
#define G4_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int g4_attn_bwd_noalloc(const g4_attn_args* args, void* stream);

/*
 * Synchronise `stream` and read the device error word of the allocation-free
 * backward's static array on the current device (the counterpart of
 * g4_read_device_error for g4_attn_bwd_noalloc, whose scratch address callers
 * never see).  *code receives 0 or a G4 device error as described there.
 */
int g4_attn_bwd_noalloc_device_error(int* code, void* stream);

/*
 * Ring context parallelism helpers (no reference counterpart: the reference
 * runs long global contexts on one GPU, h100.py:713-747).  A sequence split
 * across ranks is attended block by block of keys (g4_attn_fwd with
 * causal_shift for blocks that lie wholly before the queries); each block
 * gives its rows a partial output and LSE.
 *
 * g4_merge_attention_partial: o_acc / lse_acc (fp32 running output, natural
 * log LSE) <- the exact softmax combination with a block's bf16 output o_part
 * and its lse_part:  L = log(e^La + e^Lb), O = Oa e^(La-L) + Ob e^(Lb-L).
 * Rows with La = Lb = -inf stay O = 0, L = -inf (start from o_acc = 0,
 * lse_acc = -inf).  Output strides [token, head] in elements with unit feature
 * stride; LSE strides [head, token] in floats.
 *
 * g4_cast_f32_bf16: dst (bf16, strides [token, head]) <- src (fp32, contiguous
 * [token][head][head_dim]): the final dQ / dK / dV / O of accumulated calls.
 */
typedef struct g4_merge_args {
  float* o_acc;
  float* lse_acc;
  const void* o_part;
  const float* lse_part;
  int64_t o_acc_stride[2];
  int64_t o_part_stride[2];
  int64_t lse_acc_stride[2];
  int64_t lse_part_stride[2];
  int32_t tokens;
  int32_t heads;
  int32_t head_dim;  /* a multiple of 8 */
} g4_merge_args;
int g4_merge_attention_partial(const g4_merge_args* args, void* stream);
int g4_cast_f32_bf16(const float* src, void* dst, int64_t tokens, int32_t heads, int32_t head_dim,
                     int64_t dst_token_stride, int64_t dst_head_stride, void* stream);
/* dst += src over n floats (n a multiple of 4, 16-byte aligned): the key
 * gradients of a sliding-window halo returned to the rank that owns the keys. */
int g4_add_f32(float* dst, const float* src, int64_t n, void* stream);

/*
 * Synchronise `stream` and read the device error word of a workspace used by
 * a previous call; *code receives 0 or a G4 device error (1 = TMA wait
 * expired, 2 = MMA wait expired, 3 = role hand-off wait expired).
 */
int g4_read_device_error(const void* workspace, int* code, void* stream);

/*
 * Self-test of the bounded waits every kernel uses (no reference counterpart:
 * the reference's kernels have no wait bound).  One CTA on the current device,
 * synchronous.  mode 0: the awaited barrier completes; mode 1: nothing
 * completes it and the wait expires after the library's 2 s bound; mode 2:
 * another warp raises the CTA abort word first (recording device error 1) and
 * the wait returns at once.  Outputs: *code the device error word, *completed
 * 1 if the wait saw the barrier complete, *wait_ms the wait's duration.
 * Nothing here faults or hangs the GPU.
 */
int g4_selftest_wait(int mode, int* code, int* completed, double* wait_ms);

/*
 * Block-sparse tile schedule of a local layer (window > 0): for every query
 * tile of 128 rows (flattened over sequences / segments), the key tiles of 128
 * keys that hold at least one allowed (query, key) pair, ascending.  This is
 * the exact incidence the kernels iterate: tiles outside a list are never
 * loaded.  An entry is the key tile's index in bits 0-29; bit 31 is set when
 * every pair of the tile (valid rows and keys) is allowed, which lets the
 * kernels skip the mask there; bit 30 when no key of the tile is a vision
 * token and every valid row and key of the tile lie in one document, so the
 * window / causal range rule alone is exact there (no metadata is read).
 * Replaces build_gemma4_local_sparse_schedule / SparseTileRows
 * (src/gemma4_fa4/sparse_schedule.py:181-374, host Python in the reference;
 * built on the device here).  Outputs (device int32): counts[n_q_tiles] and
 * key_tiles[n_q_tiles * stride], stride >= ceil(max Sk / 128).  For packed
 * layouts n_q_tiles is sum over segments of ceil(len_q / 128); entries past
 * it are unspecified.  Scratch: workspace of g4_tile_schedule_workspace_bytes.
 */
size_t g4_tile_schedule_workspace_bytes(const g4_attn_args* args);
int g4_tile_schedule(const g4_attn_args* args, int32_t* counts, int32_t* key_tiles,
                     int32_t stride, void* stream);

/*
 * Dense Gemma-4 mask builder: writes out[b][q][k] = 1 if allowed, else 0
 * (uint8, (B,Sq,Sk) contiguous).  Query row i sits at absolute position
 * q_start + i (q_start < 0 selects lower-right alignment, kv_len - q_len).
 * window == 0 means no sliding window.  Replaces src/gemma4_fa4/masks.py:8-80
 * (gemma4_attention_mask); vision/document ids (int32) and key padding
 * (uint8) are (B,Sk) contiguous and nullable.
 */
int g4_build_mask(uint8_t* out, int32_t batch, int32_t q_len, int32_t kv_len, int32_t q_start,
                  int32_t window, int32_t allow_vision_bidirectional, const int32_t* vision_ids,
                  const int32_t* document_ids, const uint8_t* key_padding, void* stream);

/*
 * Fused Q/K/V preparation (rows of one projection output, bf16):
 *   rot   = RoPE(Norm(x) * weight)   Norm(x) = x * (mean(x^2) + eps)^-1/2
 *   plain = Norm(x)
 * RoPE is rotate-half on the leading rotary_dim features, the rest passed
 * through: rot_i = n_i cos_i - n_{i+h} sin_i (i < h), n_i cos_i + n_{i-h} sin_i
 * (h <= i < rotary_dim), h = rotary_dim / 2.
 * Gemma-4 uses it as Q = RoPE(QNorm(q_proj)), K = RoPE(KNorm(k_proj)),
 * V = VNorm(v_proj) (src/gemma4_fa4/h100_torch_ops.py:302-326, :396-403) and,
 * for global layers, K = partial_RoPE(KNorm(Z)), V = VNorm(Z) from one source
 * Z in a single pass (both outputs set; src/gemma4_fa4/reference.py:306-328).
 * Layer-op tables are full width (rotary_dim = head_dim) with the
 * proportional partial rotation carried by cos = 1, sin = 0 entries; the
 * reference helper's tables cover only the rotated subspace.
 * The backward applies both adjoints and sums them into dx
 * (docs/design.md:202-213), and optionally returns the FP32 gradient of the
 * learned scale, reduced deterministically through the workspace.
 */
typedef struct g4_prep_args {
  const void* x;        /* (B,S,H,head_dim), feature stride 1 */
  const void* weight;   /* learned scale (head_dim), nullable = no scale */
  const void* cos;      /* (B,S,rotary_dim), feature stride 1; unused if rotary_dim == 0 */
  const void* sin;
  void* rot;            /* forward output, nullable */
  void* plain;          /* forward output, nullable */
  const void* drot;     /* backward: cotangent of rot, nullable */
  const void* dplain;   /* backward: cotangent of plain, nullable */
  void* dx;             /* backward output */
  float* dweight;       /* backward output (head_dim floats), nullable; needs weight and drot */
  /* strides in elements: [batch, token, head], non-negative multiples of 8 */
  int64_t x_stride[3];
  int64_t rot_stride[3];
  int64_t plain_stride[3];
  int64_t drot_stride[3];
  int64_t dplain_stride[3];
  int64_t dx_stride[3];
  int64_t cos_stride[2];  /* [batch, token]; 0 broadcasts */
  int32_t batch;
  int32_t seqlen;
  int32_t num_heads;
  int32_t head_dim;     /* 256 or 512 */
  int32_t rotary_dim;   /* 0 (no rotation) or a power of two in [16, head_dim] */
  float eps;            /* 1e-6 for Gemma-4 */
  void* workspace;      /* backward with dweight: g4_prep_bwd_workspace_bytes */
  size_t workspace_bytes;
} g4_prep_args;

/* Workspace bytes of g4_prep_bwd (0 without dweight; no device access). */
size_t g4_prep_bwd_workspace_bytes(const g4_prep_args* args);
/* rot and/or plain from x.  Replaces the eager norm/rotary chain of the
 * reference layer ops (h100_torch_ops.py:396-403, :456-461, :729-733, :840-843). */
int g4_prep_fwd(const g4_prep_args* args, void* stream);
/* dx (and dweight) from drot and/or dplain; the adjoint of g4_prep_fwd
 * (torch autograd through reference.py:276-328 in the reference). */
int g4_prep_bwd(const g4_prep_args* args, void* stream);

/*
 * Launch accounting and opt-in timing (benchmark/profiling support; no
 * reference counterpart -- the reference times whole Python calls).
 * Kernel ids: 0 forward, 1 backward preprocess, 2 backward dQ (recompute),
 * 3 backward dK/dV (recompute), 4 planning (tile lists, vision pairs, tile
 * ranges), 5 mask builder, 6 backward P/dS scores, 7-9 backward dV / dK / dQ
 * tile GEMMs (materialised path), 10 two-pass forward softmax, 11 two-pass
 * forward O = P V, 12 decode, 13 decode combine, 14 preparation forward,
 * 15 preparation backward, 16 preparation dweight reduction, 17 wait self-test,
 * 18 backward dV and dK tile GEMMs in one launch (used instead of 7 and 8 when
 * the dO and Q operands take at most 80 MiB together), 19 fp32 -> bf16 cast
 * (the dV / dK of a multi-band backward), 20 ring merge of a partial output,
 * 21 fp32 add (halo key gradients), 22 short-window decode (sliding layers,
 * query groups of at most 4 heads: one launch, merge fused).
 *  - g4_launch_count: launches of `kernel_id` issued by this process so far.
 *  - g4_profile_enable(1): every later launch is bracketed by CUDA events on
 *    its own stream; g4_profile_read synchronises those events and returns the
 *    launches and summed device milliseconds per kernel id since the last
 *    g4_profile_reset.  Not for use inside CUDA graph capture.
 */
int g4_kernel_count(void);
const char* g4_kernel_name(int kernel_id);
int g4_launch_count(int kernel_id, long long* count);
int g4_profile_enable(int enable);
int g4_profile_reset(void);
int g4_profile_read(int kernel_id, long long* launches, double* total_ms);

#ifdef __cplusplus
}
#endif

#endif /* GEMMA4_B200_H_ */
