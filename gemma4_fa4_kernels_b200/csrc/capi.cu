// C-ABI layer of libgemma4_b200.so: argument validation, workspace planning,
// TMA tensor-map construction and kernel launches.  See include/gemma4_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gemma4_b200.h"
#include "g4_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(G4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------------------
// launch accounting / opt-in event timing
// ---------------------------------------------------------------------------------------
enum KernelId {
  kKFwd = 0,
  kKBwdPre,
  kKBwdDq,
  kKBwdDkv,
  kKPlan,
  kKMask,
  kKScore,
  kKGemmDv,
  kKGemmDk,
  kKGemmDq,
  kKFwdScore,
  kKFwdPv,
  kKDecode,
  kKDecodeCombine,
  kKPrepFwd,
  kKPrepBwd,
  kKPrepDw,
  kKSelftest,
  kKGemmDvDk,
  kKCast,
  kKMerge,
  kKAdd,
  kKDecodeShort,
  kKReset,
  kKCount
};
const char* const kKernelNames[kKCount] = {"attn_fwd", "bwd_preprocess", "bwd_dq", "bwd_dkv",
                                           "plan",     "mask",           "bwd_score",
                                           "bwd_gemm_dv", "bwd_gemm_dk", "bwd_gemm_dq",
                                           "fwd_score",   "fwd_pv",      "decode",
                                           "decode_combine", "prep_fwd",  "prep_bwd",
                                           "prep_dw_reduce", "selftest_wait", "bwd_gemm_dvdk",
                                           "cast_f32_bf16", "ring_merge", "add_f32",
                                           "decode_short", "workspace_reset"};
std::atomic<long long> g_launches[kKCount];
std::atomic<bool> g_profile{false};
struct ProfRecord {
  int id;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
std::vector<ProfRecord> g_prof_records;

// Brackets one launch: counts it and, when profiling, records events around it.
class LaunchScope {
 public:
  LaunchScope(int id, cudaStream_t st) : id_(id), st_(st) {
    g_launches[id].fetch_add(1);
    if (g_profile.load()) {
      if (cudaEventCreate(&a_) == cudaSuccess && cudaEventCreate(&b_) == cudaSuccess) {
        cudaEventRecord(a_, st_);
        timed_ = true;
      }
    }
  }
  ~LaunchScope() {
    if (!timed_) return;
    cudaEventRecord(b_, st_);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_records.push_back({id_, a_, b_});
  }

 private:
  int id_;
  cudaStream_t st_;
  cudaEvent_t a_{}, b_{};
  bool timed_ = false;
};

// ---------------------------------------------------------------------------------------
// TMA tensor maps (driver entry point fetched through the runtime, no -lcuda needed)
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 tensor viewed as (D, H, S, B) with a (64, 1, rows, 1) box, 128-B swizzle.
int make_map(CUtensorMap* map, const void* ptr, int64_t d, int64_t h, int64_t s, int64_t b,
             int64_t stride_h, int64_t stride_s, int64_t stride_b, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (b <= 1) stride_b = stride_s * (s > 0 ? s : 1);
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)h, (cuuint64_t)(s > 0 ? s : 1),
                        (cuuint64_t)(b > 0 ? b : 1)};
  cuuint64_t strides[3] = {(cuuint64_t)(stride_h * 2), (cuuint64_t)(stride_s * 2),
                           (cuuint64_t)(stride_b * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(G4_ERR_INVALID, "tensor map encoding failed (CUresult %d)", (int)r);
  return G4_OK;
}

// Scratch tiles viewed as bytes: (256, 64, n_half) with (256, 64, 1) boxes, one
// box per 16 KB half of a 32 KB pre-swizzled tile (copied as is, no swizzle).
int make_scratch_map(CUtensorMap* map, const void* ptr, int64_t n_half) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {256, 64, (cuuint64_t)(n_half > 0 ? n_half : 1)};
  cuuint64_t strides[2] = {256, 16384};
  cuuint32_t box[3] = {256, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(G4_ERR_INVALID, "scratch tensor map encoding failed (CUresult %d)", (int)r);
  return G4_OK;
}

// ---------------------------------------------------------------------------------------
// argument checks shared by forward and backward
// ---------------------------------------------------------------------------------------
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_strides(const int64_t* st, const char* name, bool packed) {
  for (int i = packed ? 1 : 0; i < 3; ++i)
    if (st[i] <= 0 || (st[i] % 8) != 0)
      return fail(G4_ERR_INVALID, "%s strides must be positive multiples of 8 elements", name);
  return G4_OK;
}

int check_common(const g4_attn_args* a) {
  if (!a) return fail(G4_ERR_INVALID, "null argument block");
  const bool packed = a->cu_seqlens_q != nullptr;
  if ((a->cu_seqlens_k != nullptr) != packed)
    return fail(G4_ERR_INVALID, "cu_seqlens_q and cu_seqlens_k must both be set or both be null");
  if (!a->q || !a->k || !a->v || !a->o || !a->lse)
    return fail(G4_ERR_INVALID, "q, k, v, o and lse are required");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o))
    return fail(G4_ERR_INVALID, "q, k, v and o base pointers must be 16-byte aligned");
  if (a->workspace && !aligned16(a->workspace))  // bulk copies and tensor maps of the scratch
    return fail(G4_ERR_INVALID, "workspace must be 16-byte aligned");
  if (a->k == a->v) return fail(G4_ERR_INVALID, "K and V must be distinct operands");
  if (a->batch <= 0 || a->seqlen_q <= 0 || a->seqlen_k <= 0)
    return fail(G4_ERR_INVALID, "batch and sequence lengths must be positive");
  // every query keeps q_abs = q + Sk - Sq + shift >= 0: Sq may exceed Sk only by
  // the causal shift (ring blocks whose keys all precede their queries)
  const int64_t shift = a->window == 0 ? std::max<int64_t>(0, a->causal_shift) : 0;
  if (!packed && int64_t(a->seqlen_q) > int64_t(a->seqlen_k) + shift)
    return fail(G4_ERR_UNSUPPORTED, "fixed layout requires Sq <= Sk + causal_shift");
  if (a->num_kv_heads <= 0 || a->num_q_heads <= 0 || a->num_q_heads % a->num_kv_heads)
    return fail(G4_ERR_INVALID, "query heads must be a positive multiple of KV heads");
  if (a->head_dim_qk != a->head_dim_v || (a->head_dim_qk != 256 && a->head_dim_qk != 512))
    return fail(G4_ERR_UNSUPPORTED, "head dims must be (256,256) or (512,512)");
  if (a->window < 0) return fail(G4_ERR_INVALID, "window must be >= 0");
  if (a->window == 0 && (a->vision_ids || a->document_ids))
    return fail(G4_ERR_UNSUPPORTED, "vision/document metadata applies to local layers only");
  if (a->causal_shift < 0) return fail(G4_ERR_INVALID, "causal_shift must be >= 0");
  if (a->causal_shift != 0 && a->window != 0)
    return fail(G4_ERR_UNSUPPORTED, "causal_shift applies to global layers only");
  if (a->grad_accumulate != 0 && a->grad_accumulate != 1)
    return fail(G4_ERR_INVALID, "grad_accumulate must be 0 or 1");
  int rc;
  if ((rc = check_strides(a->q_stride, "q", packed))) return rc;
  if ((rc = check_strides(a->k_stride, "k", packed))) return rc;
  if ((rc = check_strides(a->v_stride, "v", packed))) return rc;
  if ((rc = check_strides(a->o_stride, "o", packed))) return rc;
  if (packed && (a->max_seqlen_q <= 0 || a->max_seqlen_k <= 0 || a->max_seqlen_q > a->max_seqlen_k))
    return fail(G4_ERR_UNSUPPORTED, "packed maxima must satisfy 1 <= max Sq <= max Sk");
  return G4_OK;
}

// ---------------------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------------------
struct Workspace {
  size_t header = 0;       // int err, n_q_tiles, n_k_tiles
  size_t q_tiles = 0;      // int2[max_q_tiles]
  size_t k_tiles = 0;      // int2[max_k_tiles]
  size_t pair_last = 0;    // int[meta_len]
  size_t pair_first = 0;   // int[meta_len] (backward)
  size_t delta = 0;        // float[Hq * tokens_q]
  size_t lse2 = 0;         // float[Hq * tokens_q]
  // materialised-P/dS backward only
  size_t seg_first = 0;    // int[B] (packed)
  size_t ranges = 0;       // int4[n_qt_total]
  size_t klist = 0;        // metadata masks: int[n_qt_total * klist_stride] key-tile lists
  int klist_stride = 0;
  size_t p_tiles = 0;      // Hq * head_cap tiles of 32 KB
  size_t ds_tiles = 0;
  size_t fwd_alpha = 0;    // two-pass forward: float[Hq * head_cap * 128]
  size_t fwd_flags = 0;    // int[Hq * head_cap]
  size_t fwd_inv_l = 0;    // float[Hq * tokens_q]
  // single-token decode
  bool decode = false;
  int decode_splits = 0;
  size_t part_o = 0;       // float[B * Hq * splits * D]
  size_t part_ml = 0;      // float2[B * Hq * splits]
  size_t decode_counters = 0;  // int[B * Hkv] (short-window decode)
  bool materialized = false;
  int n_qt_total = 0;
  int64_t head_cap_tiles = 0;
  size_t total = 0;
  int max_q_tiles = 0;
  int max_k_tiles = 0;
  int64_t tokens_q = 0;
};

// SM count of the current device (148 on B200; also the answer when no device
// is visible, so that size queries work on hosts without a GPU).
int sm_count() {
  constexpr int kDev = 64;
  static std::atomic<int> cached[kDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDev) {
    cudaGetLastError();
    return 148;
  }
  int n = cached[dev].load();
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev].store(n);
  }
  return n;
}

// A second stream per device for the backward's dQ GEMM, which needs nothing of
// the dV / dK GEMMs: forked from the caller's stream after a band's score
// passes and joined back before the next launch, so each GEMM's last, partly
// empty wave runs beside the other's CTAs.  The fork and join events are
// shared by every call on the device, so one mutex keeps each record / wait
// pair together (calls from several host threads stay correct; their dQ
// launches are merely ordered on the one side stream).  Stream capture forks
// the side stream into the graph and the join brings it back.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr;
  cudaEvent_t join = nullptr;
};
std::mutex g_side_mu;

SideStream* side_stream() {  // call with g_side_mu held; nullptr when unavailable
  constexpr int kDev = 64;
  static SideStream side[kDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDev) {
    cudaGetLastError();
    return nullptr;
  }
  SideStream& sd = side[dev];
  if (!sd.stream) {
    cudaStream_t st = nullptr;
    cudaEvent_t f = nullptr, j = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&f, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&j, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      if (st) cudaStreamDestroy(st);
      if (f) cudaEventDestroy(f);
      return nullptr;
    }
    sd.fork = f;
    sd.join = j;
    sd.stream = st;
  }
  return &sd;
}

// One query token per sequence: the split-key decode kernels serve the call.
bool decode_eligible(const g4_attn_args* a) {
  const bool packed = a->cu_seqlens_q != nullptr;
  const int sq = packed ? a->max_seqlen_q : a->seqlen_q;
  return sq == 1 && a->num_kv_heads > 0 && a->num_q_heads % a->num_kv_heads == 0 &&
         a->num_q_heads / a->num_kv_heads <= g4::kDecodeMaxGroup;
}

// Sliding-window decode with query groups of at most four heads runs the
// short-window kernel (CUDA cores, one launch); everything else the
// tensor-core split-key kernel and its merge.
int64_t decode_keys(const g4_attn_args* a) {
  int64_t keys = a->cu_seqlens_q ? a->max_seqlen_k : a->seqlen_k;
  if (a->window > 0) keys = std::min<int64_t>(keys, a->window);
  return keys;
}

bool decode_short(const g4_attn_args* a) {
  const int G = a->num_q_heads / a->num_kv_heads;
  return a->window > 0 && G <= g4::kDecodeShortMaxGroup &&
         decode_keys(a) <=
             int64_t(g4::kDecodeShortMaxSplits) * g4::decode_short_keys(a->head_dim_qk, G);
}

// Key-range splits per (sequence, KV head).  Short-window kernel: two CTAs per
// SM, at least 32 keys and at most decode_short_keys(D, G) keys per CTA.  Tensor-core
// kernel: enough CTAs for one per SM, never more splits than 128-key tiles, and
// no split left without a tile at the longest sequence.
int decode_splits(const g4_attn_args* a) {
  const bool packed = a->cu_seqlens_q != nullptr;
  int64_t keys = packed ? a->max_seqlen_k : a->seqlen_k;
  if (a->window > 0) keys = std::min<int64_t>(keys, a->window);
  if (decode_short(a)) {
    const int64_t units = std::max<int64_t>(1, int64_t(a->batch) * a->num_kv_heads);
    const int per = g4::decode_short_keys(a->head_dim_qk, a->num_q_heads / a->num_kv_heads);
    const int64_t lo = (keys + per - 1) / per;
    // one wave: at most two CTAs per SM in total
    int64_t n = std::min<int64_t>(std::max<int64_t>(1, 2 * sm_count() / units),
                                  std::max<int64_t>(1, keys / 32));
    n = std::max<int64_t>(std::max<int64_t>(n, lo), 1);
    return static_cast<int>(std::min<int64_t>(n, g4::kDecodeShortMaxSplits));
  }
  const int64_t max_tiles = std::max<int64_t>(1, (keys + g4::kTileN - 1) / g4::kTileN);
  const int64_t units = std::max<int64_t>(1, int64_t(a->batch) * a->num_kv_heads);
  int64_t n = (sm_count() + units - 1) / units;
  n = std::max<int64_t>(1, std::min<int64_t>(std::min(n, max_tiles), g4::kDecodeMaxSplits));
  const int64_t tps = (max_tiles + n - 1) / n;
  return static_cast<int>((max_tiles + tps - 1) / tps);
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Workspace modes: 0 single-kernel forward, 1 backward with recompute kernels,
// 2 backward with materialised P/dS tiles, 3 two-pass forward (d512, P tiles).
// plan_workspace lays out the regions every mode shares (and, for modes 2/3,
// the problem-wide tile plan); the band scratch of modes 2/3 follows
// w.total (see plan_bands).  With vision / document metadata, modes 0 and 2
// also hold the exact key-tile list of every query tile (klist).
Workspace plan_workspace(const g4_attn_args* a, int mode) {
  Workspace w;
  const bool packed = a->cu_seqlens_q != nullptr;
  if ((mode == 0 || mode == 3) && decode_eligible(a)) {
    size_t off = 256;
    w.decode = true;
    w.decode_splits = decode_splits(a);
    if (decode_short(a)) {  // arrival counters of the fused merge, zeroed per call
      w.decode_counters = off;
      off = align256(off + sizeof(int) * size_t(a->batch) * size_t(a->num_kv_heads));
    }
    if (w.decode_splits > 1) {
      const size_t rows = size_t(a->batch) * size_t(a->num_q_heads) * size_t(w.decode_splits);
      w.part_o = off;
      off = align256(off + rows * size_t(a->head_dim_v) * sizeof(float));
      w.part_ml = off;
      off = align256(off + rows * 2 * sizeof(float));
    }
    w.total = off;
    return w;
  }
  const bool vision = a->vision_ids && a->window > 0;
  const bool lists = a->window > 0 && (a->vision_ids || a->document_ids);
  const bool two_pass_fwd = mode == 3 && !vision && a->head_dim_qk == 512;
  const int backward = (mode == 1 || mode == 2) ? mode : 0;
  size_t off = 256;
  if (packed) {
    w.max_q_tiles = a->seqlen_q / g4::kTileM + a->batch + 1;
    w.q_tiles = off;
    off = align256(off + sizeof(int2) * w.max_q_tiles);
    if (backward) {
      w.max_k_tiles = a->seqlen_k / g4::kTileN + a->batch + 1;
      w.k_tiles = off;
      off = align256(off + sizeof(int2) * w.max_k_tiles);
    }
  }
  if (vision) {
    const int64_t meta_len = packed ? a->seqlen_k : int64_t(a->batch) * a->seqlen_k;
    w.pair_last = off;
    off = align256(off + sizeof(int) * meta_len);
    if (backward) {
      w.pair_first = off;
      off = align256(off + sizeof(int) * meta_len);
    }
  }
  w.tokens_q = packed ? a->seqlen_q : int64_t(a->batch) * a->seqlen_q;
  if (backward) {
    w.delta = off;
    off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
    w.lse2 = off;
    off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
  }
  const bool fwd_lists = mode == 0 && lists;  // the single-kernel forward reads the lists
  if (backward == 2 || two_pass_fwd || fwd_lists) {
    w.materialized = !fwd_lists;
    w.n_qt_total = packed ? w.max_q_tiles
                          : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
    if (packed) {
      w.seg_first = off;
      off = align256(off + sizeof(int) * a->batch);
    }
    w.ranges = off;
    off = align256(off + sizeof(int4) * w.n_qt_total);
    if (lists) {
      w.klist_stride = ceil_div(packed ? a->max_seqlen_k : a->seqlen_k, g4::kTileN);
      w.klist = off;
      off = align256(off + sizeof(int) * size_t(w.n_qt_total) * w.klist_stride);
    }
    if (two_pass_fwd) {
      w.fwd_inv_l = off;
      off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
    }
  }
  w.total = off;
  return w;
}

template <typename T>
T* ws_ptr(const g4_attn_args* a, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(a->workspace) + off);
}

g4::SeqLayout make_layout(const g4_attn_args* a) {
  g4::SeqLayout l;
  l.batch = a->batch;
  l.seqlen_q = a->seqlen_q;
  l.seqlen_k = a->seqlen_k;
  l.cu_q = a->cu_seqlens_q;
  l.cu_k = a->cu_seqlens_k;
  l.meta_stride = a->seqlen_k;
  l.causal_shift = a->window == 0 ? a->causal_shift : 0;
  return l;
}

// ---------------------------------------------------------------------------------------
// materialised path: bands
// ---------------------------------------------------------------------------------------
// A band is a set of KV heads and up to two ranges of the flattened query-tile
// list whose P (and dS) tiles fit the scratch at once.  One launch set runs per
// band.  Plans, in order of preference:
//   1. one band (the whole problem; the common case);
//   2. bands of KV heads over all query tiles (every dV / dK still complete);
//   3. bands of query tiles over all heads: a band takes tiles from the end of
//      the list (long causal rows) and from its start (short rows), so every
//      band is a mix that keeps the SMs evenly loaded; dV / dK are partial per
//      band and summed in fp32 (TMA reduce-add), then converted once.
struct Band {
  int g[4];
  int h0, nh;          // KV heads
  int kv_item0, kv_items;  // key-major grid (items are key tiles)
  int rows;            // query tiles in the band
};

struct MatPlan {
  bool ok = false;
  bool acc_kv = false;   // the dV / dK products add fp32 (caller accumulators or own_acc)
  bool own_acc = false;  // fp32 dV / dK buffers in the workspace, cast to bf16 at the end
  int64_t cap = 0;     // scratch tiles per query head of a band
  int nh_max = 0;
  size_t p_off = 0, ds_off = 0, alpha_off = 0, flags_off = 0, dk_acc_off = 0, dv_acc_off = 0;
  size_t total = 0;
  std::vector<Band> bands;
};

// Per query tile of the problem: key-tile range, count and sequence; per
// sequence: the key-major index of its first key tile.
struct TileTable {
  std::vector<int> kt_lo, n_kt, seq;
  std::vector<int> kfirst;  // packed: first key-tile list index of each segment (+ end)
  int nk_per_seq = 0;       // fixed: key tiles per sequence
  bool lists = false;       // counts of listed key tiles (not ranges): kt_lo + n_kt - 1 is no bound
  bool exact = false;
};

// Key-tile range of one query tile (text masks; the planner kernel's rule).
void qtile_range(int len_q, int len_k, int qt, int window, int shift, int* kt_lo, int* n_kt) {
  const int q_off = len_k - len_q + shift;
  const int qa0 = qt * g4::kTileM + q_off;
  const int qa1 = std::min((qt + 1) * g4::kTileM, len_q) - 1 + q_off;
  const int lo = window > 0 ? std::max(0, qa0 - window + 1) : 0;
  const int hi = std::min(qa1, len_k - 1);
  *kt_lo = hi >= lo ? lo / g4::kTileN : 0;
  *n_kt = hi >= lo ? hi / g4::kTileN - lo / g4::kTileN + 1 : 0;
}

// Exact table from the sequence lengths (host copies).
void table_from_lengths(const g4_attn_args* a, const std::vector<int>& len_q,
                        const std::vector<int>& len_k, TileTable* t) {
  const int shift = a->window == 0 ? a->causal_shift : 0;
  const bool packed = a->cu_seqlens_q != nullptr;
  t->kt_lo.clear();
  t->n_kt.clear();
  t->seq.clear();
  t->kfirst.assign(len_q.size() + 1, 0);
  for (size_t s = 0; s < len_q.size(); ++s) {
    const int nqt = ceil_div(len_q[s], g4::kTileM);
    for (int qt = 0; qt < nqt; ++qt) {
      int lo, n;
      qtile_range(len_q[s], len_k[s], qt, a->window, shift, &lo, &n);
      t->kt_lo.push_back(lo);
      t->n_kt.push_back(n);
      t->seq.push_back(static_cast<int>(s));
    }
    t->kfirst[s + 1] = t->kfirst[s] + ceil_div(len_k[s], g4::kTileN);
  }
  t->nk_per_seq = packed ? 0 : ceil_div(a->seqlen_k, g4::kTileN);
  t->exact = true;
}

// Upper bound of the problem's scratch tiles per query head, from arguments
// alone (no device access): exact for fixed layouts.
int64_t bound_tiles(const g4_attn_args* a, int n_qt_total) {
  const bool packed = a->cu_seqlens_q != nullptr;
  if (a->window > 0 && (a->vision_ids || a->document_ids))  // listed tiles: up to every key tile
    return int64_t(ceil_div(packed ? a->max_seqlen_k : a->seqlen_k, g4::kTileN)) * n_qt_total;
  if (packed) {
    const int64_t kmax = ceil_div(a->max_seqlen_k, g4::kTileN);
    int64_t per = kmax;
    if (a->window > 0) per = std::min<int64_t>(per, (a->window + 126) / g4::kTileN + 2);
    return per * n_qt_total;
  }
  TileTable t;
  std::vector<int> lq(1, a->seqlen_q), lk(1, a->seqlen_k);
  table_from_lengths(a, lq, lk, &t);
  int64_t total = 0;
  for (int n : t.n_kt) total += n;
  return total * a->batch;
}

// Bytes per scratch tile and query head: P + dS (backward) or P + its row
// rescale factors + the tile flag (two-pass forward).
size_t tile_bytes(bool backward) {
  return backward ? 2 * 32768 : 32768 + 128 * sizeof(float) + sizeof(int);
}

// Places a band plan's regions after the shared prefix.
void place(const g4_attn_args* a, const Workspace& w, bool backward, MatPlan* m) {
  const int G = a->num_q_heads / a->num_kv_heads;
  const size_t heads = size_t(m->nh_max) * G;
  const size_t tiles = heads * size_t(m->cap);
  size_t off = w.total;
  if (m->own_acc) {
    const int64_t tok_k = a->cu_seqlens_q ? a->seqlen_k : int64_t(a->batch) * a->seqlen_k;
    const size_t acc = size_t(tok_k) * a->num_kv_heads * a->head_dim_qk * sizeof(float);
    m->dk_acc_off = off;
    off = align256(off + acc);
    m->dv_acc_off = off;
    off = align256(off + acc);
  }
  m->p_off = off;
  off = align256(off + tiles * 32768);
  if (backward) {
    m->ds_off = off;
    off = align256(off + tiles * 32768);
  } else {
    m->alpha_off = off;
    off = align256(off + tiles * 128 * sizeof(float));
    m->flags_off = off;
    off = align256(off + tiles * sizeof(int));
  }
  m->total = off;
}

// Single-band size (the *_workspace_bytes queries): every tile of the bound.
size_t single_band_bytes(const g4_attn_args* a, const Workspace& w, bool backward) {
  MatPlan m;
  m.nh_max = a->num_kv_heads;
  m.cap = bound_tiles(a, w.n_qt_total);
  place(a, w, backward, &m);
  return m.total;
}

// Key-major grid of a band: the key tiles its query tiles reach.
void band_kv_items(const g4_attn_args* a, const TileTable& t, Band* b) {
  const bool packed = a->cu_seqlens_q != nullptr;
  int lo = INT32_MAX, hi = -1;
  for (int r = 0; r < 2; ++r)
    for (int g = b->g[2 * r]; g < b->g[2 * r + 1]; ++g) {
      if (t.n_kt[g] <= 0) continue;
      const int s = t.seq[g];
      const int first = packed ? t.kfirst[s] + t.kt_lo[g] : t.kt_lo[g];
      int last = packed ? t.kfirst[s] + t.kt_lo[g] + t.n_kt[g] - 1 : t.kt_lo[g] + t.n_kt[g] - 1;
      if (t.lists) last = packed ? t.kfirst[s + 1] - 1 : t.nk_per_seq - 1;
      lo = std::min(lo, first);
      hi = std::max(hi, last);
    }
  if (hi < lo) {
    b->kv_item0 = 0;
    b->kv_items = 0;
  } else if (packed) {
    b->kv_item0 = lo;
    b->kv_items = hi - lo + 1;
  } else {  // fixed items run key tile major: item = tile * B + sequence
    b->kv_item0 = lo * a->batch;
    b->kv_items = (hi - lo + 1) * a->batch;
  }
}

// Query-tile bands of capacity `cap` tiles per head (see the comment above).
std::vector<Band> qtile_bands(const TileTable& t, int64_t cap, int h0, int nh) {
  std::vector<Band> out;
  const int n = static_cast<int>(t.n_kt.size());
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    Band b;
    b.h0 = h0;
    b.nh = nh;
    b.g[0] = b.g[1] = lo;
    b.g[2] = b.g[3] = hi + 1;
    int64_t sum = 0;
    // long rows from the end (at least one tile), up to half the capacity
    while (hi >= lo && (b.g[2] == b.g[3] || sum + t.n_kt[hi] <= cap / 2)) {
      sum += t.n_kt[hi];
      --hi;
      b.g[2] = hi + 1;
    }
    while (lo <= hi && sum + t.n_kt[lo] <= cap) {  // short rows from the start
      sum += t.n_kt[lo];
      ++lo;
      b.g[1] = lo;
    }
    while (hi >= lo && sum + t.n_kt[hi] <= cap) {  // room left: more from the end
      sum += t.n_kt[hi];
      --hi;
      b.g[2] = hi + 1;
    }
    out.push_back(b);
  }
  return out;
}

// Band plan for a workspace of `ws_bytes`; `t` must be exact unless one band
// of the bound fits.  Returns false when no band fits (then the compact
// kernels run).
bool plan_bands(const g4_attn_args* a, const Workspace& w, bool backward, size_t ws_bytes,
                const TileTable* t, bool accumulate, MatPlan* m) {
  const int G = a->num_q_heads / a->num_kv_heads;
  const int Hkv = a->num_kv_heads;
  const size_t per = tile_bytes(backward);
  const size_t avail = ws_bytes > w.total ? ws_bytes - w.total : 0;
  m->bands.clear();
  m->ok = false;
  m->acc_kv = accumulate;
  auto full_band = [&](int h0, int nh) {
    Band b;
    b.g[0] = 0;
    b.g[1] = w.n_qt_total;
    b.g[2] = b.g[3] = w.n_qt_total;
    b.h0 = h0;
    b.nh = nh;
    b.rows = w.n_qt_total;
    // every key tile (zeros for keys no query reaches)
    const int nk = a->cu_seqlens_q ? w.max_k_tiles
                                   : a->batch * ceil_div(a->seqlen_k, g4::kTileN);
    b.kv_item0 = 0;
    b.kv_items = nk;
    return b;
  };
  // 1. one band over the bound
  const int64_t bound = bound_tiles(a, w.n_qt_total);
  {
    MatPlan c;
    c.acc_kv = accumulate;
    c.nh_max = Hkv;
    c.cap = bound;
    place(a, w, backward, &c);
    if (c.total <= ws_bytes && bound > 0) {
      *m = c;
      m->bands.push_back(full_band(0, Hkv));
      m->ok = true;
      return true;
    }
  }
  if (!t || !t->exact) return false;
  int64_t total = 0, widest = 0;
  for (int n : t->n_kt) {
    total += n;
    widest = std::max<int64_t>(widest, n);
  }
  if (total == 0) return false;
  // 2. bands of KV heads
  {
    const int nh = static_cast<int>(
        std::min<int64_t>(Hkv, avail / std::max<size_t>(1, size_t(G) * size_t(total) * per)));
    if (nh >= 1) {
      MatPlan c;
      c.acc_kv = accumulate;
      c.nh_max = nh;
      c.cap = total;
      place(a, w, backward, &c);
      if (c.total <= ws_bytes) {
        *m = c;
        for (int h0 = 0; h0 < Hkv; h0 += nh) {
          Band b = full_band(h0, std::min(nh, Hkv - h0));
          if (accumulate) band_kv_items(a, *t, &b);
          m->bands.push_back(b);
        }
        m->ok = true;
        return true;
      }
    }
  }
  // 3. bands of query tiles (dV / dK summed in fp32: into the caller's
  // accumulators, or into workspace buffers converted at the end)
  MatPlan c;
  c.acc_kv = backward;
  c.own_acc = backward && !accumulate;
  for (int nh = Hkv; nh >= 1; nh = nh > 1 ? nh / 2 : 0) {
    if (Hkv % nh) continue;
    c.nh_max = nh;
    c.cap = 0;
    place(a, w, backward, &c);  // fixed regions (accumulators) with an empty scratch
    const size_t left = ws_bytes > c.total ? ws_bytes - c.total : 0;
    const int64_t cap = static_cast<int64_t>(left / (size_t(nh) * G * per)) - 2;  // alignment slack
    if (cap < widest) continue;
    c.cap = cap;
    place(a, w, backward, &c);
    if (c.total > ws_bytes) continue;
    *m = c;
    for (int h0 = 0; h0 < Hkv; h0 += nh)
      for (Band b : qtile_bands(*t, cap, h0, nh)) {
        b.rows = (b.g[1] - b.g[0]) + (b.g[3] - b.g[2]);
        band_kv_items(a, *t, &b);
        m->bands.push_back(b);
      }
    m->ok = true;
    return true;
  }
  return false;
}

// Zeroes a call's workspace header (and the short-window decode's arrival
// counters): `bytes` (a multiple of 16) at a 16-byte aligned `words`, by one CTA
// instead of a memset.  It triggers griddepcontrol.launch_dependents at once, so
// the call's first kernel (a chained launch) is dispatched while it runs; that
// kernel waits for it (pdl_enter) before touching the header: at its start for
// the attention kernels, only before its first counter access for the
// short-window decode, whose loads and arithmetic overlap it.  A plain launch,
// it starts after every earlier kernel of the stream has completed.
__global__ void __launch_bounds__(256) workspace_reset_kernel(int4* words, int n) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int i = threadIdx.x; i < n; i += blockDim.x) words[i] = make_int4(0, 0, 0, 0);
}

int reset_workspace(void* words, size_t bytes, cudaStream_t st) {
  LaunchScope ls(kKReset, st);
  workspace_reset_kernel<<<1, 256, 0, st>>>(static_cast<int4*>(words),
                                             static_cast<int>(bytes / sizeof(int4)));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? G4_OK : cuda_fail(e, "workspace reset");
}

// Common prologue: zero the header, plan packed tiles and metadata bounds.
int prepare(const g4_attn_args* a, const Workspace& w, bool backward, cudaStream_t st,
            g4::MaskSpec* mask) {
  if (!a->workspace || a->workspace_bytes < w.total)
    return fail(G4_ERR_WORKSPACE, "workspace of %zu bytes required", w.total);
  if (int rc = reset_workspace(a->workspace, 256, st)) return rc;
  const g4::SeqLayout layout = make_layout(a);
  int* hdr = ws_ptr<int>(a, 0);
  if (a->cu_seqlens_q) {
    LaunchScope ls(kKPlan, st);
    int rc = g4::launch_plan_tiles(a->cu_seqlens_q, a->batch, g4::kTileM,
                                   ws_ptr<int2>(a, w.q_tiles), hdr + 1,
                                   w.seg_first ? ws_ptr<int>(a, w.seg_first) : nullptr, st);
    if (rc) return cuda_fail(static_cast<cudaError_t>(rc), "q tile planning");
    if (backward) {
      LaunchScope ls2(kKPlan, st);
      rc = g4::launch_plan_tiles(a->cu_seqlens_k, a->batch, g4::kTileN,
                                 ws_ptr<int2>(a, w.k_tiles), hdr + 2, nullptr, st);
      if (rc) return cuda_fail(static_cast<cudaError_t>(rc), "k tile planning");
    }
  }
  mask->window = a->window;
  mask->vis = a->window > 0 ? a->vision_ids : nullptr;
  mask->doc = a->window > 0 ? a->document_ids : nullptr;
  mask->pair_last = nullptr;
  mask->pair_first = nullptr;
  if (w.pair_last) {
    int* pl = ws_ptr<int>(a, w.pair_last);
    int* pf = w.pair_first ? ws_ptr<int>(a, w.pair_first) : nullptr;
    LaunchScope ls(kKPlan, st);
    int rc = g4::launch_pair_last(layout, a->vision_ids, a->document_ids, pl, pf, a->batch, st);
    if (rc) return cuda_fail(static_cast<cudaError_t>(rc), "vision pair planning");
    mask->pair_last = pl;
    mask->pair_first = pf;
  }
  return G4_OK;
}

// Exact tile table for a band plan.  Fixed layouts: from the arguments.
// Packed layouts: the segment lengths are read back from the device (one
// stream synchronisation, as the reference's host-side schedule also reads
// cu_seqlens); not possible while the stream is being captured.
int exact_table(const g4_attn_args* a, cudaStream_t st, TileTable* t) {
  if (!a->cu_seqlens_q) {
    std::vector<int> lq(a->batch, a->seqlen_q), lk(a->batch, a->seqlen_k);
    table_from_lengths(a, lq, lk, t);
    return G4_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    t->exact = false;
    return G4_OK;
  }
  std::vector<int> cq(a->batch + 1), ck(a->batch + 1);
  cudaError_t e = cudaMemcpyAsync(cq.data(), a->cu_seqlens_q, sizeof(int) * cq.size(),
                                  cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ck.data(), a->cu_seqlens_k, sizeof(int) * ck.size(),
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cu_seqlens read-back");
  std::vector<int> lq(a->batch), lk(a->batch);
  for (int s = 0; s < a->batch; ++s) {
    lq[s] = cq[s + 1] - cq[s];
    lk[s] = ck[s + 1] - ck[s];
    if (lq[s] < 0 || lk[s] < 0 || lq[s] > lk[s])
      return fail(G4_ERR_INVALID, "cu_seqlens must be non-decreasing with Sq <= Sk per segment");
  }
  table_from_lengths(a, lq, lk, t);
  return G4_OK;
}

// Exact table from the device plan (metadata masks: listed key tiles per query
// tile): the ranges written by the planners and, for packed layouts, the key
// lengths are read back (one stream synchronisation, as the reference's
// host-side schedule also builds its lists on the host); not possible while
// the stream is being captured.
int table_from_device(const g4_attn_args* a, const Workspace& w, cudaStream_t st, TileTable* t) {
  t->exact = false;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return G4_OK;
  }
  const bool packed = a->cu_seqlens_q != nullptr;
  int hdr[4] = {0, 0, 0, 0};
  std::vector<int4> rg(w.n_qt_total);
  std::vector<int> ck(packed ? a->batch + 1 : 0);
  cudaError_t e = cudaMemcpyAsync(hdr, a->workspace, sizeof(hdr), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(rg.data(), ws_ptr<int4>(a, w.ranges), sizeof(int4) * rg.size(),
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && packed)
    e = cudaMemcpyAsync(ck.data(), a->cu_seqlens_k, sizeof(int) * ck.size(),
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "tile plan read-back");
  const int n = packed ? std::min(hdr[1], w.n_qt_total) : w.n_qt_total;
  t->kt_lo.resize(n);
  t->n_kt.resize(n);
  t->seq.resize(n);
  for (int g = 0; g < n; ++g) {
    t->kt_lo[g] = rg[g].x;
    t->n_kt[g] = rg[g].y;
    t->seq[g] = rg[g].w;
  }
  if (packed) {
    t->kfirst.assign(a->batch + 1, 0);
    for (int s2 = 0; s2 < a->batch; ++s2)
      t->kfirst[s2 + 1] = t->kfirst[s2] + ceil_div(std::max(0, ck[s2 + 1] - ck[s2]), g4::kTileN);
  }
  t->nk_per_seq = packed ? 0 : ceil_div(a->seqlen_k, g4::kTileN);
  t->lists = true;
  t->exact = true;
  return G4_OK;
}

g4::MatParams mat_band(g4::MatParams m, const Band& b) {
  for (int i = 0; i < 4; ++i) m.band_g[i] = b.g[i];
  m.band_h0 = b.h0;
  m.band_nh = b.nh;
  m.kv_item0 = b.kv_item0;
  return m;
}

// fp32 (D, H, S, B) view for the accumulators, (32, 1, 128, 1) boxes, 128-B swizzle.
int make_map_f32(CUtensorMap* map, const void* ptr, int64_t d, int64_t h, int64_t s, int64_t b,
                 int64_t stride_h, int64_t stride_s, int64_t stride_b) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (b <= 1) stride_b = stride_s * (s > 0 ? s : 1);
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)h, (cuuint64_t)(s > 0 ? s : 1),
                        (cuuint64_t)(b > 0 ? b : 1)};
  cuuint64_t strides[3] = {(cuuint64_t)(stride_h * 4), (cuuint64_t)(stride_s * 4),
                           (cuuint64_t)(stride_b * 4)};
  cuuint32_t box[4] = {32, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(G4_ERR_INVALID, "fp32 tensor map encoding failed (CUresult %d)", (int)r);
  return G4_OK;
}

// Single-token decode: split-key kernel, then the merge of the splits.
int run_decode(const g4_attn_args* a, cudaStream_t st) {
  const Workspace w = plan_workspace(a, 0);
  if (!a->workspace || a->workspace_bytes < w.total)
    return fail(G4_ERR_WORKSPACE, "workspace of %zu bytes required", w.total);
  const bool short_kernel = decode_short(a);
  // header, and the short kernel's arrival counters right behind it
  const size_t reset = short_kernel ? align256(w.decode_counters + sizeof(int) * size_t(a->batch) *
                                                                   size_t(a->num_kv_heads))
                                    : 256;
  if (int rc = reset_workspace(a->workspace, reset, st)) return rc;
  const bool packed = a->cu_seqlens_q != nullptr;
  g4::DecodeParams p;
  memset(&p, 0, sizeof(p));
  p.layout = make_layout(a);
  p.window = a->window;
  p.doc = a->window > 0 ? a->document_ids : nullptr;
  p.group = a->num_q_heads / a->num_kv_heads;
  p.num_q_heads = a->num_q_heads;
  p.n_split = w.decode_splits;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.o = static_cast<__nv_bfloat16*>(a->o);
  for (int i = 0; i < 3; ++i) {
    p.q_stride[i] = a->q_stride[i];
    p.o_stride[i] = a->o_stride[i];
  }
  p.lse = a->lse;
  p.lse_stride[0] = packed ? 0 : a->lse_stride[0];
  p.lse_stride[1] = packed ? a->seqlen_q : a->lse_stride[1];
  p.part_o = w.part_o ? ws_ptr<float>(a, w.part_o) : nullptr;
  p.part_ml = w.part_ml ? ws_ptr<float2>(a, w.part_ml) : nullptr;
  p.err = ws_ptr<int>(a, 0);
  const int D = a->head_dim_qk;
  if (short_kernel) {
    p.k = static_cast<const __nv_bfloat16*>(a->k);
    p.v = static_cast<const __nv_bfloat16*>(a->v);
    for (int i = 0; i < 3; ++i) {
      p.k_stride[i] = packed && i == 0 ? 0 : a->k_stride[i];
      p.v_stride[i] = packed && i == 0 ? 0 : a->v_stride[i];
    }
    p.counters = ws_ptr<int>(a, w.decode_counters);
    LaunchScope ls(kKDecodeShort, st);
    const int e = g4::launch_decode_short(D, p, a->num_kv_heads, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "short-window decode launch");
    return G4_OK;
  }
  const int64_t bk = packed ? 1 : a->batch;
  CUtensorMap tk, tv;
  int rc;
  if ((rc = make_map(&tk, a->k, D, a->num_kv_heads, a->seqlen_k, bk, a->k_stride[2],
                     a->k_stride[1], a->k_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tv, a->v, a->head_dim_v, a->num_kv_heads, a->seqlen_k, bk, a->v_stride[2],
                     a->v_stride[1], a->v_stride[0], 128)))
    return rc;
  {
    LaunchScope ls(kKDecode, st);
    const int e = g4::launch_decode(D, tk, tv, p, a->num_kv_heads, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "decode launch");
  }
  if (p.n_split > 1) {
    LaunchScope ls(kKDecodeCombine, st);
    const int e = g4::launch_decode_combine(D, p, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "decode combine launch");
  }
  return G4_OK;
}

// Scratch for g4_attn_bwd_noalloc: a fixed-size static device array instead of
// a caller-provided workspace.  In host code the symbol is only a host-side
// stand-in, never a device address; noalloc_scratch() asks the runtime for the
// array's address on the current device.  The lookup runs on every call (it is
// cheap), so an address never outlives the context it was taken in (a device
// reset or a re-created primary context gets a fresh one).
static __device__ __align__(256) uint8_t g_noalloc_scratch[G4_NOALLOC_SCRATCH_BYTES];

int noalloc_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
  *out = p;
  return G4_OK;
}

}  // namespace

extern "C" {

int g4_abi_version(void) { return G4_ABI_VERSION; }

const char* g4_last_error(void) { return g_last_error.c_str(); }

size_t g4_attn_fwd_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  const Workspace w = plan_workspace(args, 3);
  return w.materialized ? single_band_bytes(args, w, false) : w.total;
}

size_t g4_attn_fwd_min_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  return plan_workspace(args, 0).total;
}

size_t g4_attn_bwd_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  const Workspace w = plan_workspace(args, 2);
  return w.materialized ? single_band_bytes(args, w, true) : w.total;
}

size_t g4_attn_bwd_min_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  return plan_workspace(args, 1).total;
}

int g4_attn_fwd(const g4_attn_args* a, void* stream) {
  g_last_error.clear();
  int rc = check_common(a);
  if (rc) return rc;
  const bool packed = a->cu_seqlens_q != nullptr;
  if (!packed && (a->lse_stride[0] <= 0 || a->lse_stride[1] <= 0))
    return fail(G4_ERR_INVALID, "lse strides must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (decode_eligible(a)) return run_decode(a, st);
  // Two-pass d512 forward (P tiles in HBM, no QK^T recomputation), one launch
  // pair per band, when the workspace holds one band's scratch; otherwise the
  // single-kernel forward.
  const Workspace w3 = plan_workspace(a, 3);
  MatPlan mp;
  if (w3.materialized && a->workspace && a->workspace_bytes >= w3.total) {
    if (!plan_bands(a, w3, false, a->workspace_bytes, nullptr, false, &mp)) {
      TileTable t;
      if ((rc = exact_table(a, st, &t))) return rc;
      plan_bands(a, w3, false, a->workspace_bytes, &t, false, &mp);
    }
  }
  const Workspace w = mp.ok ? w3 : plan_workspace(a, 0);
  g4::FwdParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = prepare(a, w, false, st, &p.mask))) return rc;
  p.layout = make_layout(a);
  p.group = a->num_q_heads / a->num_kv_heads;
  p.o = static_cast<__nv_bfloat16*>(a->o);
  for (int i = 0; i < 3; ++i) p.o_stride[i] = a->o_stride[i];
  p.lse = a->lse;
  p.lse_stride[0] = packed ? 0 : a->lse_stride[0];
  p.lse_stride[1] = packed ? a->seqlen_q : a->lse_stride[1];
  p.err = ws_ptr<int>(a, 0);
  if (packed) {
    p.tiles = ws_ptr<int2>(a, w.q_tiles);
    p.n_tiles = ws_ptr<int>(a, 0) + 1;
  }
  const int D = a->head_dim_qk;
  const int64_t bq = packed ? 1 : a->batch;
  CUtensorMap tq, tk, tv;
  if ((rc = make_map(&tq, a->q, D, a->num_q_heads, a->seqlen_q, bq, a->q_stride[2], a->q_stride[1],
                     a->q_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tk, a->k, D, a->num_kv_heads, a->seqlen_k, bq, a->k_stride[2],
                     a->k_stride[1], a->k_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tv, a->v, a->head_dim_v, a->num_kv_heads, a->seqlen_k, bq, a->v_stride[2],
                     a->v_stride[1], a->v_stride[0], 64)))
    return rc;
  const int grid_x = packed ? w.max_q_tiles
                            : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
  if (mp.ok) {
    g4::MatParams m;
    memset(&m, 0, sizeof(m));
    m.layout = p.layout;
    m.mask = p.mask;
    m.group = p.group;
    m.num_q_heads = a->num_q_heads;
    m.n_qt_fixed = packed ? 0 : (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
    m.q_tiles = p.tiles;
    m.n_q_tiles = p.n_tiles;
    m.ranges = ws_ptr<int4>(a, w.ranges);
    m.head_cap_tiles = mp.cap;
    m.p_tiles = ws_ptr<uint8_t>(a, mp.p_off);
    m.fwd_alpha = ws_ptr<float>(a, mp.alpha_off);
    m.fwd_flags = ws_ptr<int>(a, mp.flags_off);
    m.fwd_inv_l = ws_ptr<float>(a, w.fwd_inv_l);
    m.ws_head_stride = w.tokens_q;
    m.lse_out = a->lse;
    m.lse_stride[0] = p.lse_stride[0];
    m.lse_stride[1] = p.lse_stride[1];
    m.o = p.o;
    for (int i = 0; i < 3; ++i) m.o_stride[i] = p.o_stride[i];
    m.err = p.err;
    CUtensorMap tv64;
    if ((rc = make_map(&tv64, a->v, a->head_dim_v, a->num_kv_heads, a->seqlen_k, bq,
                       a->v_stride[2], a->v_stride[1], a->v_stride[0], 64)))
      return rc;
    CUtensorMap to128;  // O, written by TMA stores in 128-row tiles
    if ((rc = make_map(&to128, a->o, a->head_dim_v, a->num_q_heads, a->seqlen_q, bq,
                       a->o_stride[2], a->o_stride[1], a->o_stride[0], 128)))
      return rc;
    CUtensorMap tp;  // the P scratch as bytes: the d512 O = P V GEMM runs as CTA pairs
    const bool pairs = g4::gemm_pairs_ok(D, 3, m);
    if (pairs && (rc = make_scratch_map(&tp, m.p_tiles,
                                        2 * int64_t(mp.nh_max) * p.group * mp.cap)))
      return rc;
    int e;
    {
      LaunchScope ls(kKPlan, st);
      e = g4::launch_plan_qtile_ranges(m, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "query-tile range planning");
    }
    for (const Band& b : mp.bands) {
      const g4::MatParams mb = mat_band(m, b);
      {
        LaunchScope ls(kKFwdScore, st);
        e = g4::launch_bwd_score(D, 2, tq, tk, tv, tq, mb, b.rows, st);
        if (e) return cuda_fail(static_cast<cudaError_t>(e), "forward score launch");
      }
      LaunchScope ls(kKFwdPv, st);
      e = g4::launch_bwd_tile_gemm(D, 3, tv64, to128, pairs ? &tp : nullptr, mb, b.rows,
                                   b.nh * p.group, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "forward PV launch");
    }
    return G4_OK;
  }
  if (w.klist) {
    // metadata masks: the exact key-tile list of every query tile first
    g4::MatParams m;
    memset(&m, 0, sizeof(m));
    m.layout = p.layout;
    m.mask = p.mask;
    m.group = p.group;
    m.num_q_heads = a->num_q_heads;
    m.n_qt_fixed = packed ? 0 : (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
    m.q_tiles = p.tiles;
    m.n_q_tiles = p.n_tiles;
    m.ranges = ws_ptr<int4>(a, w.ranges);
    m.klist = ws_ptr<int>(a, w.klist);
    m.klist_stride = w.klist_stride;
    LaunchScope ls(kKPlan, st);
    const int e = g4::launch_plan_qtile_lists(m, w.n_qt_total, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "key-tile list planning");
    p.ranges = m.ranges;
    p.klist = m.klist;
    p.klist_stride = m.klist_stride;
  }
  const int slabs = a->head_dim_v / 256;
  LaunchScope ls(kKFwd, st);
  int e;
  if (D == 256 && slabs == 1 && (p.klist != nullptr || (!p.mask.vis && !p.mask.doc))) {
    // d256: one persistent CTA per SM walks every (head, query tile) item;
    // text masks need no list, metadata masks read the planner's lists
    const int64_t items = int64_t(a->num_q_heads) * grid_x;
    const int ctas = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(items, sm_count())));
    e = g4::launch_fwd_persistent(tq, tk, tv, p, ctas, a->num_q_heads, st);
  } else {
    e = D == 256 ? g4::launch_fwd<256>(tq, tk, tv, p, grid_x, a->num_q_heads, slabs, st)
                 : g4::launch_fwd<512>(tq, tk, tv, p, grid_x, a->num_q_heads, slabs, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "forward launch");
  return G4_OK;
}

int g4_attn_bwd(const g4_attn_args* a, void* stream) {
  g_last_error.clear();
  int rc = check_common(a);
  if (rc) return rc;
  const bool packed = a->cu_seqlens_q != nullptr;
  if (!a->dout || !a->dq || !a->dk || !a->dv)
    return fail(G4_ERR_INVALID, "dout, dq, dk and dv are required");
  if (!aligned16(a->dout) || !aligned16(a->dq) || !aligned16(a->dk) || !aligned16(a->dv))
    return fail(G4_ERR_INVALID, "dout, dq, dk and dv base pointers must be 16-byte aligned");
  if ((rc = check_strides(a->do_stride, "dout", packed))) return rc;
  if ((rc = check_strides(a->dq_stride, "dq", packed))) return rc;
  if ((rc = check_strides(a->dk_stride, "dk", packed))) return rc;
  if ((rc = check_strides(a->dv_stride, "dv", packed))) return rc;
  if (!packed && (a->lse_stride[0] <= 0 || a->lse_stride[1] <= 0))
    return fail(G4_ERR_INVALID, "lse strides must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool accumulate = a->grad_accumulate != 0;
  // Materialised P/dS, band by band, when the workspace holds one band's
  // scratch; otherwise the recompute kernels (small workspaces).  With
  // vision / document metadata the tile counts are data-dependent: when the
  // bound does not fit one band, the plan is made after the device planners
  // have listed the tiles (`defer`).
  const bool lists = a->window > 0 && (a->vision_ids || a->document_ids);
  const Workspace wm = plan_workspace(a, 2);
  MatPlan mp;
  bool defer = false;
  if (wm.materialized && a->workspace && a->workspace_bytes >= wm.total) {
    if (!plan_bands(a, wm, true, a->workspace_bytes, nullptr, accumulate, &mp)) {
      if (lists) {
        defer = true;
      } else {
        TileTable t;
        if ((rc = exact_table(a, st, &t))) return rc;
        plan_bands(a, wm, true, a->workspace_bytes, &t, accumulate, &mp);
      }
    }
  }
  if (accumulate && !mp.ok && !defer)
    return fail(G4_ERR_WORKSPACE,
                "gradient accumulation runs on the materialised backward only; the workspace "
                "(%zu bytes) holds no band of its scratch",
                a->workspace_bytes);
  // the recompute kernels use the same leading regions (tile lists, vision
  // pairs, delta, log2 LSE), so a deferred plan that fails can still fall back
  const Workspace w = (mp.ok || defer) ? wm : plan_workspace(a, 1);
  g4::BwdParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = prepare(a, w, true, st, &p.mask))) return rc;
  p.layout = make_layout(a);
  p.group = a->num_q_heads / a->num_kv_heads;
  p.num_q_heads = a->num_q_heads;
  p.o = static_cast<const __nv_bfloat16*>(a->o);
  p.dout = static_cast<const __nv_bfloat16*>(a->dout);
  p.dq = static_cast<__nv_bfloat16*>(a->dq);
  p.dk = static_cast<__nv_bfloat16*>(a->dk);
  p.dv = static_cast<__nv_bfloat16*>(a->dv);
  for (int i = 0; i < 3; ++i) {
    p.o_stride[i] = a->o_stride[i];
    p.do_stride[i] = a->do_stride[i];
    p.dq_stride[i] = a->dq_stride[i];
    p.dk_stride[i] = a->dk_stride[i];
    p.dv_stride[i] = a->dv_stride[i];
  }
  p.lse = a->lse;
  p.dlse = a->dlse;
  p.lse_stride[0] = packed ? 0 : a->lse_stride[0];
  p.lse_stride[1] = packed ? a->seqlen_q : a->lse_stride[1];
  p.delta = ws_ptr<float>(a, w.delta);
  p.lse2 = ws_ptr<float>(a, w.lse2);
  p.ws_head_stride = w.tokens_q;
  p.err = ws_ptr<int>(a, 0);
  if (packed) {
    p.q_tiles = ws_ptr<int2>(a, w.q_tiles);
    p.n_q_tiles = ws_ptr<int>(a, 0) + 1;
    p.k_tiles = ws_ptr<int2>(a, w.k_tiles);
    p.n_k_tiles = ws_ptr<int>(a, 0) + 2;
  }
  int e;
  {
    LaunchScope ls(kKBwdPre, st);
    // the range planner follows at once when the band plan is made and the
    // layout is fixed without key-tile lists (it then waits late, see there)
    const bool early = (mp.ok || defer) && !packed && !lists;
    e = g4::launch_bwd_preprocess(p, a->head_dim_v, w.tokens_q, early, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "backward preprocess launch");
  const int D = a->head_dim_qk;
  const int64_t bq = packed ? 1 : a->batch;
  CUtensorMap tq, tk, tk64, tv, tdo;
  if ((rc = make_map(&tq, a->q, D, a->num_q_heads, a->seqlen_q, bq, a->q_stride[2], a->q_stride[1],
                     a->q_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tk, a->k, D, a->num_kv_heads, a->seqlen_k, bq, a->k_stride[2],
                     a->k_stride[1], a->k_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tk64, a->k, D, a->num_kv_heads, a->seqlen_k, bq, a->k_stride[2],
                     a->k_stride[1], a->k_stride[0], 64)))
    return rc;
  if ((rc = make_map(&tv, a->v, a->head_dim_v, a->num_kv_heads, a->seqlen_k, bq, a->v_stride[2],
                     a->v_stride[1], a->v_stride[0], 128)))
    return rc;
  if ((rc = make_map(&tdo, a->dout, a->head_dim_v, a->num_q_heads, a->seqlen_q, bq,
                     a->do_stride[2], a->do_stride[1], a->do_stride[0], 128)))
    return rc;
  const int gq = packed ? w.max_q_tiles : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
  const int gk = packed ? w.max_k_tiles : a->batch * ((a->seqlen_k + g4::kTileN - 1) / g4::kTileN);
  if (mp.ok || defer) {
    g4::MatParams m;
    memset(&m, 0, sizeof(m));
    m.layout = p.layout;
    m.mask = p.mask;
    m.group = p.group;
    m.num_q_heads = a->num_q_heads;
    m.n_qt_fixed = packed ? 0 : (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
    m.q_tiles = p.q_tiles;
    m.n_q_tiles = p.n_q_tiles;
    m.k_tiles = p.k_tiles;
    m.n_k_tiles = p.n_k_tiles;
    m.seg_first_qtile = packed ? ws_ptr<int>(a, w.seg_first) : nullptr;
    m.ranges = ws_ptr<int4>(a, w.ranges);
    m.klist = lists ? ws_ptr<int>(a, w.klist) : nullptr;
    m.klist_stride = w.klist_stride;
    {
      if (lists) {
        LaunchScope ls(kKPlan, st);
        e = g4::launch_plan_qtile_lists(m, w.n_qt_total, st);
        if (e) return cuda_fail(static_cast<cudaError_t>(e), "key-tile list planning");
      }
      LaunchScope ls(kKPlan, st);
      e = g4::launch_plan_qtile_ranges(m, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "query-tile range planning");
    }
    if (defer) {
      TileTable t;
      if ((rc = table_from_device(a, w, st, &t))) return rc;
      if (t.exact) plan_bands(a, wm, true, a->workspace_bytes, &t, accumulate, &mp);
      if (!mp.ok && accumulate)
        return fail(G4_ERR_WORKSPACE,
                    "gradient accumulation runs on the materialised backward only; the "
                    "workspace (%zu bytes) holds no band of its scratch",
                    a->workspace_bytes);
    }
  }
  if (mp.ok) {
    g4::MatParams m;
    memset(&m, 0, sizeof(m));
    m.layout = p.layout;
    m.mask = p.mask;
    m.group = p.group;
    m.num_q_heads = a->num_q_heads;
    m.n_qt_fixed = packed ? 0 : (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
    m.q_tiles = p.q_tiles;
    m.n_q_tiles = p.n_q_tiles;
    m.k_tiles = p.k_tiles;
    m.n_k_tiles = p.n_k_tiles;
    m.seg_first_qtile = packed ? ws_ptr<int>(a, w.seg_first) : nullptr;
    m.ranges = ws_ptr<int4>(a, w.ranges);
    m.klist = lists ? ws_ptr<int>(a, w.klist) : nullptr;
    m.klist_stride = w.klist_stride;
    m.head_cap_tiles = mp.cap;
    m.p_tiles = ws_ptr<uint8_t>(a, mp.p_off);
    m.ds_tiles = ws_ptr<uint8_t>(a, mp.ds_off);
    m.lse2 = p.lse2;
    m.delta = p.delta;
    m.ws_head_stride = p.ws_head_stride;
    m.dq = p.dq;
    m.dk = p.dk;
    m.dv = p.dv;
    for (int i = 0; i < 3; ++i) {
      m.dq_stride[i] = p.dq_stride[i];
      m.dk_stride[i] = p.dk_stride[i];
      m.dv_stride[i] = p.dv_stride[i];
    }
    m.err = p.err;
    const int Hkv = a->num_kv_heads;
    const int64_t tok_k = packed ? a->seqlen_k : int64_t(a->batch) * a->seqlen_k;
    // fp32 destinations: the caller's accumulators, or the band sums of dV / dK
    m.acc_q = accumulate ? 1 : 0;
    m.acc_kv = mp.acc_kv ? 1 : 0;
    if (accumulate) {
      m.dq_acc = static_cast<float*>(a->dq);
      m.dk_acc = static_cast<float*>(a->dk);
      m.dv_acc = static_cast<float*>(a->dv);
      for (int i = 0; i < 3; ++i) {
        m.dq_acc_stride[i] = a->dq_stride[i];
        m.dk_acc_stride[i] = a->dk_stride[i];
        m.dv_acc_stride[i] = a->dv_stride[i];
      }
    } else if (mp.own_acc) {
      m.dk_acc = ws_ptr<float>(a, mp.dk_acc_off);
      m.dv_acc = ws_ptr<float>(a, mp.dv_acc_off);
      const int64_t st_acc[3] = {packed ? 0 : int64_t(a->seqlen_k) * Hkv * D, int64_t(Hkv) * D, D};
      for (int i = 0; i < 3; ++i) m.dk_acc_stride[i] = m.dv_acc_stride[i] = st_acc[i];
    }
    CUtensorMap tq64, tdo64;
    if ((rc = make_map(&tq64, a->q, D, a->num_q_heads, a->seqlen_q, bq, a->q_stride[2],
                       a->q_stride[1], a->q_stride[0], 64)))
      return rc;
    if ((rc = make_map(&tdo64, a->dout, a->head_dim_v, a->num_q_heads, a->seqlen_q, bq,
                       a->do_stride[2], a->do_stride[1], a->do_stride[0], 64)))
      return rc;
    // gradients: bf16 TMA stores in 128-row tiles, or fp32 reduce-adds
    CUtensorMap tdq, tdk, tdv;
    if (accumulate) {
      if ((rc = make_map_f32(&tdq, a->dq, D, a->num_q_heads, a->seqlen_q, bq, a->dq_stride[2],
                             a->dq_stride[1], a->dq_stride[0])))
        return rc;
    } else if ((rc = make_map(&tdq, a->dq, D, a->num_q_heads, a->seqlen_q, bq, a->dq_stride[2],
                              a->dq_stride[1], a->dq_stride[0], 128))) {
      return rc;
    }
    if (mp.acc_kv) {
      if ((rc = make_map_f32(&tdk, m.dk_acc, D, Hkv, a->seqlen_k, bq, m.dk_acc_stride[2],
                             m.dk_acc_stride[1], m.dk_acc_stride[0])))
        return rc;
      if ((rc = make_map_f32(&tdv, m.dv_acc, a->head_dim_v, Hkv, a->seqlen_k, bq,
                             m.dv_acc_stride[2], m.dv_acc_stride[1], m.dv_acc_stride[0])))
        return rc;
    } else {
      if ((rc = make_map(&tdk, a->dk, D, Hkv, a->seqlen_k, bq, a->dk_stride[2], a->dk_stride[1],
                         a->dk_stride[0], 128)))
        return rc;
      if ((rc = make_map(&tdv, a->dv, a->head_dim_v, Hkv, a->seqlen_k, bq, a->dv_stride[2],
                         a->dv_stride[1], a->dv_stride[0], 128)))
        return rc;
    }
    CUtensorMap tds;  // the dS scratch as bytes: the d512 dQ GEMM runs as CTA pairs
    const bool pairs = g4::gemm_pairs_ok(D, 2, m);
    if (pairs && (rc = make_scratch_map(&tds, m.ds_tiles,
                                        2 * int64_t(mp.nh_max) * p.group * mp.cap)))
      return rc;
    if (mp.own_acc) {
      const size_t acc = size_t(tok_k) * Hkv * D * sizeof(float);
      cudaError_t ce = cudaMemsetAsync(m.dk_acc, 0, acc, st);
      if (ce == cudaSuccess) ce = cudaMemsetAsync(m.dv_acc, 0, acc, st);
      if (ce != cudaSuccess) return cuda_fail(ce, "accumulator reset");
    }
    // dV and dK in one launch evens out the end of the KV-major grid, but it
    // streams both B operands (dO and Q) at once: only when together they take
    // at most 80 MiB of the 126 MB L2 (measured: 64 MiB, -12%; 256 MiB, no gain).
    const int64_t b_bytes =
        int64_t(w.tokens_q) * a->num_q_heads * (int64_t(D) + a->head_dim_v) * 2;
    for (const Band& b : mp.bands) {
      const g4::MatParams mb = mat_band(m, b);
      for (int pass = 0; pass < (D == 512 ? 2 : 1); ++pass) {
        LaunchScope ls(kKScore, st);
        e = g4::launch_bwd_score(D, pass, tq, tk, tv, tdo, mb, b.rows, st);
        if (e) return cuda_fail(static_cast<cudaError_t>(e), "score launch");
      }
      // dQ on the side stream, forked after the score passes, joined after dV / dK
      // (serialised on the caller's stream while launches are being profiled, so
      // that every launch's events time that kernel alone)
      std::unique_lock<std::mutex> side_lock(g_side_mu);
      SideStream* sd = g_profile.load() ? nullptr : side_stream();
      if (sd && (cudaEventRecord(sd->fork, st) != cudaSuccess ||
                 cudaStreamWaitEvent(sd->stream, sd->fork, 0) != cudaSuccess)) {
        cudaGetLastError();
        sd = nullptr;  // dQ stays on the caller's stream
      }
      {
        cudaStream_t sq = sd ? sd->stream : st;
        LaunchScope ls(kKGemmDq, sq);
        e = g4::launch_bwd_tile_gemm(D, 2, tk64, tdq, pairs ? &tds : nullptr, mb, b.rows,
                                     b.nh * p.group, sq);
        if (!e && sd) e = static_cast<int>(cudaEventRecord(sd->join, sd->stream));
        if (e) {
          if (sd) cudaStreamWaitEvent(st, sd->join, 0);
          return cuda_fail(static_cast<cudaError_t>(e), "dQ launch");
        }
      }
      if (b.kv_items > 0) {
        if (b_bytes <= (int64_t(80) << 20)) {
          LaunchScope ls(kKGemmDvDk, st);
          e = g4::launch_bwd_tile_gemm_dvdk(D, tdo64, tdv, tq64, tdk, mb, b.kv_items, b.nh, st);
        } else {
          {
            LaunchScope ls(kKGemmDv, st);
            e = g4::launch_bwd_tile_gemm(D, 0, tdo64, tdv, nullptr, mb, b.kv_items, b.nh, st);
          }
          if (!e) {
            LaunchScope ls(kKGemmDk, st);
            e = g4::launch_bwd_tile_gemm(D, 1, tq64, tdk, nullptr, mb, b.kv_items, b.nh, st);
          }
        }
      }
      if (sd) {
        const cudaError_t je = cudaStreamWaitEvent(st, sd->join, 0);  // join before any return
        if (!e && je != cudaSuccess) e = static_cast<int>(je);
      }
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "dV/dK launch");
    }
    if (mp.own_acc) {
      const int64_t rows_b = a->seqlen_k;  // packed: one "batch" of Tk rows
      {
        LaunchScope ls(kKCast, st);
        e = g4::launch_cast_f32_bf16(m.dk_acc, tok_k, Hkv, D, p.dk, a->dk_stride, a->batch,
                                     rows_b, st);
        if (e) return cuda_fail(static_cast<cudaError_t>(e), "dK cast launch");
      }
      LaunchScope ls(kKCast, st);
      e = g4::launch_cast_f32_bf16(m.dv_acc, tok_k, Hkv, a->head_dim_v, p.dv, a->dv_stride,
                                   a->batch, rows_b, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "dV cast launch");
    }
    return G4_OK;
  }
  {
    LaunchScope ls(kKBwdDq, st);
    e = D == 256 ? g4::launch_bwd_dq<256>(tq, tk, tk64, tv, tdo, p, gq, st)
                 : g4::launch_bwd_dq<512>(tq, tk, tk64, tv, tdo, p, gq, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "dQ launch");
  {
    LaunchScope ls(kKBwdDkv, st);
    e = D == 256 ? g4::launch_bwd_dkv<256>(tq, tk, tv, tdo, p, gk, st)
                 : g4::launch_bwd_dkv<512>(tq, tk, tv, tdo, p, gk, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "dK/dV launch");
  return G4_OK;
}

// Key-tile schedule of a local layer: the lists the attention kernels iterate.
namespace {
Workspace schedule_workspace(const g4_attn_args* a) {
  Workspace w = plan_workspace(a, 0);
  if (!w.klist) {  // text masks: the kernels use ranges; list them the same way here
    const bool packed = a->cu_seqlens_q != nullptr;
    w.n_qt_total = packed ? w.max_q_tiles
                          : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
    size_t off = w.total;
    w.ranges = off;
    off = align256(off + sizeof(int4) * w.n_qt_total);
    w.klist_stride = ceil_div(packed ? a->max_seqlen_k : a->seqlen_k, g4::kTileN);
    w.klist = off;
    off = align256(off + sizeof(int) * size_t(w.n_qt_total) * w.klist_stride);
    w.total = off;
  }
  return w;
}
}  // namespace

size_t g4_tile_schedule_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  return schedule_workspace(args).total;
}

int g4_tile_schedule(const g4_attn_args* a, int32_t* counts, int32_t* key_tiles, int32_t stride,
                     void* stream) {
  g_last_error.clear();
  // geometry only: the schedule depends on lengths and metadata, not on operands
  if (!a) return fail(G4_ERR_INVALID, "null argument block");
  const bool pk = a->cu_seqlens_q != nullptr;
  if ((a->cu_seqlens_k != nullptr) != pk)
    return fail(G4_ERR_INVALID, "cu_seqlens_q and cu_seqlens_k must both be set or both be null");
  if (a->batch <= 0 || a->seqlen_q <= 0 || a->seqlen_k <= 0)
    return fail(G4_ERR_INVALID, "batch and sequence lengths must be positive");
  if (!pk && a->seqlen_q > a->seqlen_k)
    return fail(G4_ERR_UNSUPPORTED, "fixed layout requires Sq <= Sk");
  if (pk && (a->max_seqlen_q <= 0 || a->max_seqlen_k <= 0 || a->max_seqlen_q > a->max_seqlen_k))
    return fail(G4_ERR_UNSUPPORTED, "packed maxima must satisfy 1 <= max Sq <= max Sk");
  if (a->window <= 0) return fail(G4_ERR_UNSUPPORTED, "tile schedules describe local layers");
  int rc;
  if (!counts || !key_tiles) return fail(G4_ERR_INVALID, "counts and key_tiles are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Workspace w = schedule_workspace(a);
  if (stride < w.klist_stride)
    return fail(G4_ERR_INVALID, "stride must be at least %d (key tiles of the longest sequence)",
                w.klist_stride);
  g4::MaskSpec mask;
  if ((rc = prepare(a, w, false, st, &mask))) return rc;
  const bool packed = a->cu_seqlens_q != nullptr;
  g4::MatParams m;
  memset(&m, 0, sizeof(m));
  m.layout = make_layout(a);
  m.mask = mask;
  m.group = a->num_q_heads / a->num_kv_heads;
  m.num_q_heads = a->num_q_heads;
  m.n_qt_fixed = packed ? 0 : (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
  m.q_tiles = packed ? ws_ptr<int2>(a, w.q_tiles) : nullptr;
  m.n_q_tiles = packed ? ws_ptr<int>(a, 0) + 1 : nullptr;
  m.ranges = ws_ptr<int4>(a, w.ranges);
  m.klist = key_tiles;
  m.klist_stride = stride;
  {
    LaunchScope ls(kKPlan, st);
    const int e = g4::launch_plan_qtile_lists(m, w.n_qt_total, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "key-tile list planning");
  }
  cudaError_t e = cudaMemcpy2DAsync(counts, sizeof(int32_t), &ws_ptr<int4>(a, w.ranges)->y,
                                    sizeof(int4), sizeof(int32_t), w.n_qt_total,
                                    cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "schedule count copy");
  return G4_OK;
}

int g4_attn_bwd_noalloc(const g4_attn_args* a, void* stream) {
  g_last_error.clear();
  int rc = check_common(a);  // sizes are computed from validated arguments only
  if (rc) return rc;
  const size_t need = plan_workspace(a, 1).total;
  if (need > G4_NOALLOC_SCRATCH_BYTES)
    return fail(G4_ERR_WORKSPACE,
                "this backward needs at least %zu bytes of scratch; the allocation-free entry "
                "point has %u bytes (use g4_attn_bwd with a caller workspace)",
                need, G4_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  g4_attn_args local = *a;
  local.workspace = scratch;
  local.workspace_bytes = G4_NOALLOC_SCRATCH_BYTES;
  return g4_attn_bwd(&local, stream);
}

int g4_attn_bwd_noalloc_device_error(int* code, void* stream) {
  if (!code) return fail(G4_ERR_INVALID, "code is required");
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return g4_read_device_error(scratch, code, stream);
}

// ---------------------------------------------------------------------------------------
// fused Q/K/V preparation
// ---------------------------------------------------------------------------------------
}  // extern "C"

namespace {

constexpr int kPrepMaxCtasPerSm = 8;  // 256-thread CTAs: the SM's 2048-thread limit

// Rows with extent > 1 must not overlap: sorted by stride, each stride covers
// the span of the dimensions inside it (innermost: the head_dim features).
bool prep_nonoverlapping(const int64_t* st, const int64_t* ext, int64_t d) {
  int64_t s[3], e[3];
  int n = 0;
  for (int i = 0; i < 3; ++i)
    if (ext[i] > 1) {
      s[n] = st[i];
      e[n] = ext[i];
      ++n;
    }
  for (int i = 1; i < n; ++i)
    for (int j = i; j > 0 && s[j] < s[j - 1]; --j) {
      std::swap(s[j], s[j - 1]);
      std::swap(e[j], e[j - 1]);
    }
  int64_t span = d;
  for (int i = 0; i < n; ++i) {
    if (s[i] < span) return false;
    span = s[i] * e[i];
  }
  return true;
}

int prep_check_tensor(const void* ptr, const int64_t* st, const g4_prep_args* a, const char* name,
                      bool output) {
  if (!aligned16(ptr)) return fail(G4_ERR_INVALID, "%s must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0 || (st[i] % 8) != 0)
      return fail(G4_ERR_INVALID, "%s strides must be non-negative multiples of 8 elements", name);
  if (output) {
    const int64_t ext[3] = {a->batch, a->seqlen, a->num_heads};
    if (!prep_nonoverlapping(st, ext, a->head_dim))
      return fail(G4_ERR_INVALID, "%s rows overlap", name);
  }
  return G4_OK;
}

int prep_check(const g4_prep_args* a, bool backward) {
  if (!a) return fail(G4_ERR_INVALID, "null argument block");
  if (a->batch < 0 || a->seqlen < 0 || a->num_heads < 0)
    return fail(G4_ERR_INVALID, "batch, seqlen and num_heads must be non-negative");
  if (static_cast<int64_t>(a->batch) * a->seqlen * a->num_heads > INT32_MAX)
    return fail(G4_ERR_UNSUPPORTED, "batch * seqlen * num_heads must be below 2^31 rows");
  if (a->head_dim != 256 && a->head_dim != 512)
    return fail(G4_ERR_UNSUPPORTED, "head_dim %d is not a Gemma-4 head dimension (256 or 512)",
                a->head_dim);
  if (a->rotary_dim < 0 || a->rotary_dim > a->head_dim || (a->rotary_dim % 2) != 0)
    return fail(G4_ERR_INVALID, "rotary_dim must be an even integer in [0, head_dim]");
  if (a->rotary_dim != 0 && (a->rotary_dim < 16 || (a->rotary_dim & (a->rotary_dim - 1)) != 0))
    return fail(G4_ERR_UNSUPPORTED, "rotary_dim must be 0 or a power of two >= 16");
  if (!(a->eps > 0.f) || a->eps > 1.f) return fail(G4_ERR_INVALID, "eps must be in (0, 1]");
  if (!a->x) return fail(G4_ERR_INVALID, "x is required");
  int rc = prep_check_tensor(a->x, a->x_stride, a, "x", false);
  if (rc) return rc;
  if (a->weight && !aligned16(a->weight)) return fail(G4_ERR_INVALID, "weight must be 16-byte aligned");
  const bool uses_rot = backward ? a->drot != nullptr : a->rot != nullptr;
  if (uses_rot && a->rotary_dim > 0) {
    if (!a->cos || !a->sin) return fail(G4_ERR_INVALID, "cos and sin are required when rotary_dim > 0");
    if (!aligned16(a->cos) || !aligned16(a->sin))
      return fail(G4_ERR_INVALID, "cos and sin must be 16-byte aligned");
    if (a->cos_stride[0] < 0 || a->cos_stride[1] < 0 || (a->cos_stride[0] % 8) != 0 ||
        (a->cos_stride[1] % 8) != 0)
      return fail(G4_ERR_INVALID, "cos/sin strides must be non-negative multiples of 8 elements");
  }
  if (!backward) {
    if (!a->rot && !a->plain) return fail(G4_ERR_INVALID, "at least one of rot and plain is required");
    if (a->rot && (rc = prep_check_tensor(a->rot, a->rot_stride, a, "rot", true))) return rc;
    if (a->plain && (rc = prep_check_tensor(a->plain, a->plain_stride, a, "plain", true))) return rc;
    if (a->rot && a->plain && a->rot == a->plain)
      return fail(G4_ERR_INVALID, "rot and plain must be distinct");
    return G4_OK;
  }
  if (!a->drot && !a->dplain) return fail(G4_ERR_INVALID, "at least one of drot and dplain is required");
  if (!a->dx) return fail(G4_ERR_INVALID, "dx is required");
  if (a->drot && (rc = prep_check_tensor(a->drot, a->drot_stride, a, "drot", false))) return rc;
  if (a->dplain && (rc = prep_check_tensor(a->dplain, a->dplain_stride, a, "dplain", false))) return rc;
  if ((rc = prep_check_tensor(a->dx, a->dx_stride, a, "dx", true))) return rc;
  if (a->dweight && (!a->weight || !a->drot))
    return fail(G4_ERR_INVALID, "dweight needs weight and drot");
  return G4_OK;
}

size_t prep_workspace(const g4_prep_args* a) {
  if (!a || !a->dweight) return 0;
  const int64_t rows = static_cast<int64_t>(a->batch) * a->seqlen * a->num_heads;
  const int64_t need = (rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(sm_count()) * kPrepMaxCtasPerSm;
  const int64_t grid = std::max<int64_t>(1, std::min(need, cap));
  return static_cast<size_t>(grid) * a->head_dim * sizeof(float);
}

g4::PrepParams prep_params(const g4_prep_args* a) {
  g4::PrepParams p{};
  p.batch = a->batch;
  p.seqlen = a->seqlen;
  p.heads = a->num_heads;
  p.head_dim = a->head_dim;
  p.rotary_dim = a->rotary_dim;
  p.rows = static_cast<uint32_t>(static_cast<int64_t>(a->batch) * a->seqlen * a->num_heads);
  p.div_heads = g4::prep_fastdiv(static_cast<uint32_t>(std::max(a->num_heads, 1)));
  p.div_seqlen = g4::prep_fastdiv(static_cast<uint32_t>(std::max(a->seqlen, 1)));
  p.eps = a->eps;
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.w = static_cast<const __nv_bfloat16*>(a->weight);
  p.cos = static_cast<const __nv_bfloat16*>(a->cos);
  p.sin = static_cast<const __nv_bfloat16*>(a->sin);
  p.rot = static_cast<__nv_bfloat16*>(a->rot);
  p.plain = static_cast<__nv_bfloat16*>(a->plain);
  p.drot = static_cast<const __nv_bfloat16*>(a->drot);
  p.dplain = static_cast<const __nv_bfloat16*>(a->dplain);
  p.dx = static_cast<__nv_bfloat16*>(a->dx);
  for (int i = 0; i < 3; ++i) {
    p.x_stride[i] = a->x_stride[i];
    p.rot_stride[i] = a->rot_stride[i];
    p.plain_stride[i] = a->plain_stride[i];
    p.drot_stride[i] = a->drot_stride[i];
    p.dplain_stride[i] = a->dplain_stride[i];
    p.dx_stride[i] = a->dx_stride[i];
  }
  p.cs_stride[0] = a->cos_stride[0];
  p.cs_stride[1] = a->cos_stride[1];
  return p;
}

}  // namespace

extern "C" {

size_t g4_prep_bwd_workspace_bytes(const g4_prep_args* a) { return prep_workspace(a); }

int g4_prep_fwd(const g4_prep_args* a, void* stream) {
  g_last_error.clear();
  int rc = prep_check(a, false);
  if (rc) return rc;
  const int64_t rows = static_cast<int64_t>(a->batch) * a->seqlen * a->num_heads;
  if (rows == 0) return G4_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  g4::PrepParams p = prep_params(a);
  if (!a->rot) p.rotary_dim = 0;
  const int grid = g4::prep_grid(false, p, sm_count());
  int e;
  {
    LaunchScope ls(kKPrepFwd, st);
    e = g4::launch_prep_fwd(p, grid, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "prep forward launch");
  return G4_OK;
}

int g4_prep_bwd(const g4_prep_args* a, void* stream) {
  g_last_error.clear();
  int rc = prep_check(a, true);
  if (rc) return rc;
  const size_t need = prep_workspace(a);
  if (need > 0 && (!a->workspace || a->workspace_bytes < need))
    return fail(G4_ERR_WORKSPACE, "prep backward needs %zu workspace bytes, got %zu", need,
                a->workspace ? a->workspace_bytes : (size_t)0);
  if (a->workspace && !aligned16(a->workspace))
    return fail(G4_ERR_INVALID, "workspace must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = static_cast<int64_t>(a->batch) * a->seqlen * a->num_heads;
  if (rows == 0) {
    if (a->dweight) {
      cudaError_t ce = cudaMemsetAsync(a->dweight, 0, a->head_dim * sizeof(float), st);
      if (ce != cudaSuccess) return cuda_fail(ce, "dweight clear");
    }
    return G4_OK;
  }
  g4::PrepParams p = prep_params(a);
  if (!a->drot) p.rotary_dim = 0;
  p.dw_part = a->dweight ? static_cast<float*>(a->workspace) : nullptr;
  const int grid = g4::prep_grid(true, p, sm_count());
  if (a->dweight && static_cast<size_t>(grid) * a->head_dim * sizeof(float) > need)
    return fail(G4_ERR_WORKSPACE, "prep backward grid exceeds the planned workspace");
  int e;
  {
    LaunchScope ls(kKPrepBwd, st);
    e = g4::launch_prep_bwd(p, grid, st);
  }
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "prep backward launch");
  if (a->dweight) {
    LaunchScope ls(kKPrepDw, st);
    e = g4::launch_prep_dw_reduce(p.dw_part, grid, a->head_dim, a->dweight, st);
    if (e) return cuda_fail(static_cast<cudaError_t>(e), "prep dweight reduction launch");
  }
  return G4_OK;
}

int g4_kernel_count(void) { return kKCount; }

const char* g4_kernel_name(int id) { return (id >= 0 && id < kKCount) ? kKernelNames[id] : ""; }

int g4_launch_count(int id, long long* count) {
  if (id < 0 || id >= kKCount || !count) return fail(G4_ERR_INVALID, "bad kernel id");
  *count = g_launches[id].load();
  return G4_OK;
}

int g4_profile_enable(int enable) {
  g_profile.store(enable != 0);
  return G4_OK;
}

int g4_profile_reset(void) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof_records) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  g_prof_records.clear();
  return G4_OK;
}

int g4_profile_read(int id, long long* launches, double* total_ms) {
  if (id < 0 || id >= kKCount || !launches || !total_ms) return fail(G4_ERR_INVALID, "bad kernel id");
  std::lock_guard<std::mutex> lk(g_prof_mu);
  long long n = 0;
  double ms = 0.0;
  for (auto& r : g_prof_records) {
    if (r.id != id) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "profile event");
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "profile elapsed time");
    ms += t;
    ++n;
  }
  *launches = n;
  *total_ms = ms;
  return G4_OK;
}

int g4_selftest_wait(int mode, int* code, int* completed, double* wait_ms) {
  if (mode < 0 || mode > 2 || !code || !completed || !wait_ms)
    return fail(G4_ERR_INVALID, "selftest mode must be 0, 1 or 2 and every output is required");
  void* dev = nullptr;
  cudaError_t e = cudaMalloc(&dev, 64);
  if (e != cudaSuccess) return cuda_fail(e, "selftest buffer");
  int* err = static_cast<int*>(dev);
  auto* out = reinterpret_cast<unsigned long long*>(static_cast<char*>(dev) + 16);
  e = cudaMemset(dev, 0, 64);
  int rc = 0;
  if (e == cudaSuccess) {
    LaunchScope ls(kKSelftest, nullptr);
    rc = g4::launch_selftest_wait(mode, err, out, nullptr);
  }
  if (e == cudaSuccess && rc == 0) e = cudaDeviceSynchronize();
  unsigned long long host[2] = {0, 0};
  if (e == cudaSuccess && rc == 0) e = cudaMemcpy(code, err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && rc == 0) e = cudaMemcpy(host, out, sizeof(host), cudaMemcpyDeviceToHost);
  cudaFree(dev);
  if (rc) return cuda_fail(static_cast<cudaError_t>(rc), "selftest launch");
  if (e != cudaSuccess) return cuda_fail(e, "selftest");
  *completed = static_cast<int>(host[0]);
  *wait_ms = static_cast<double>(host[1]) * 1e-6;
  return G4_OK;
}

int g4_merge_attention_partial(const g4_merge_args* a, void* stream) {
  g_last_error.clear();
  if (!a || !a->o_acc || !a->lse_acc || !a->o_part || !a->lse_part)
    return fail(G4_ERR_INVALID, "o_acc, lse_acc, o_part and lse_part are required");
  if (a->tokens < 0 || a->heads <= 0 || a->head_dim <= 0 || a->head_dim % 8)
    return fail(G4_ERR_INVALID, "tokens >= 0, heads > 0 and head_dim a positive multiple of 8");
  if (!aligned16(a->o_acc) || !aligned16(a->o_part))
    return fail(G4_ERR_INVALID, "o_acc and o_part must be 16-byte aligned");
  for (int i = 0; i < 2; ++i)
    if (a->o_acc_stride[i] % 4 || a->o_part_stride[i] % 8)
      return fail(G4_ERR_INVALID, "output strides must keep every row 16-byte aligned");
  g4::MergeParams p;
  p.o_acc = a->o_acc;
  p.lse_acc = a->lse_acc;
  p.o_part = static_cast<const __nv_bfloat16*>(a->o_part);
  p.lse_part = a->lse_part;
  for (int i = 0; i < 2; ++i) {
    p.o_acc_stride[i] = a->o_acc_stride[i];
    p.o_part_stride[i] = a->o_part_stride[i];
    p.lse_acc_stride[i] = a->lse_acc_stride[i];
    p.lse_part_stride[i] = a->lse_part_stride[i];
  }
  p.tokens = a->tokens;
  p.heads = a->heads;
  p.head_dim = a->head_dim;
  LaunchScope ls(kKMerge, static_cast<cudaStream_t>(stream));
  const int e = g4::launch_merge_partial(p, static_cast<cudaStream_t>(stream));
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "merge launch");
  return G4_OK;
}

int g4_cast_f32_bf16(const float* src, void* dst, int64_t tokens, int32_t heads, int32_t head_dim,
                     int64_t dst_token_stride, int64_t dst_head_stride, void* stream) {
  g_last_error.clear();
  if (!src || !dst) return fail(G4_ERR_INVALID, "src and dst are required");
  if (tokens < 0 || heads <= 0 || head_dim <= 0 || head_dim % 8)
    return fail(G4_ERR_INVALID, "tokens >= 0, heads > 0 and head_dim a positive multiple of 8");
  if (!aligned16(src) || !aligned16(dst) || dst_token_stride % 8 || dst_head_stride % 8)
    return fail(G4_ERR_INVALID, "src/dst must be 16-byte aligned with strides multiples of 8");
  const int64_t st[3] = {0, dst_token_stride, dst_head_stride};
  LaunchScope ls(kKCast, static_cast<cudaStream_t>(stream));
  const int e = g4::launch_cast_f32_bf16(src, tokens, heads, head_dim,
                                         static_cast<__nv_bfloat16*>(dst), st, 1,
                                         std::max<int64_t>(tokens, 1),
                                         static_cast<cudaStream_t>(stream));
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "cast launch");
  return G4_OK;
}

int g4_add_f32(float* dst, const float* src, int64_t n, void* stream) {
  g_last_error.clear();
  if (!dst || !src || n < 0 || n % 4 || !aligned16(dst) || !aligned16(src))
    return fail(G4_ERR_INVALID, "dst/src 16-byte aligned and n a non-negative multiple of 4");
  LaunchScope ls(kKAdd, static_cast<cudaStream_t>(stream));
  const int e = g4::launch_add_f32(dst, src, n, static_cast<cudaStream_t>(stream));
  if (e) return cuda_fail(static_cast<cudaError_t>(e), "add launch");
  return G4_OK;
}

int g4_read_device_error(const void* workspace, int* code, void* stream) {
  if (!workspace || !code) return fail(G4_ERR_INVALID, "workspace and code are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  e = cudaMemcpy(code, workspace, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "error word read");
  return G4_OK;
}

}  // extern "C"
