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
  kKCount
};
const char* const kKernelNames[kKCount] = {"attn_fwd", "bwd_preprocess", "bwd_dq", "bwd_dkv",
                                           "plan",     "mask",           "bwd_score",
                                           "bwd_gemm_dv", "bwd_gemm_dk", "bwd_gemm_dq",
                                           "fwd_score",   "fwd_pv",      "decode",
                                           "decode_combine", "prep_fwd",  "prep_bwd",
                                           "prep_dw_reduce", "selftest_wait", "bwd_gemm_dvdk"};
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
  if (a->k == a->v) return fail(G4_ERR_INVALID, "K and V must be distinct operands");
  if (a->batch <= 0 || a->seqlen_q <= 0 || a->seqlen_k <= 0)
    return fail(G4_ERR_INVALID, "batch and sequence lengths must be positive");
  if (!packed && a->seqlen_q > a->seqlen_k)
    return fail(G4_ERR_UNSUPPORTED, "fixed layout requires Sq <= Sk");
  if (a->num_kv_heads <= 0 || a->num_q_heads <= 0 || a->num_q_heads % a->num_kv_heads)
    return fail(G4_ERR_INVALID, "query heads must be a positive multiple of KV heads");
  if (a->head_dim_qk != a->head_dim_v || (a->head_dim_qk != 256 && a->head_dim_qk != 512))
    return fail(G4_ERR_UNSUPPORTED, "head dims must be (256,256) or (512,512)");
  if (a->window < 0) return fail(G4_ERR_INVALID, "window must be >= 0");
  if (a->window == 0 && (a->vision_ids || a->document_ids))
    return fail(G4_ERR_UNSUPPORTED, "vision/document metadata applies to local layers only");
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

// One query token per sequence: the split-key decode kernels serve the call.
bool decode_eligible(const g4_attn_args* a) {
  const bool packed = a->cu_seqlens_q != nullptr;
  const int sq = packed ? a->max_seqlen_q : a->seqlen_q;
  return sq == 1 && a->num_kv_heads > 0 && a->num_q_heads % a->num_kv_heads == 0 &&
         a->num_q_heads / a->num_kv_heads <= g4::kDecodeMaxGroup;
}

// Key-range splits per (sequence, KV head): enough CTAs for one per SM, never
// more splits than 128-key tiles, and no split left without a tile at the
// longest sequence.
int decode_splits(const g4_attn_args* a) {
  const bool packed = a->cu_seqlens_q != nullptr;
  int64_t keys = packed ? a->max_seqlen_k : a->seqlen_k;
  if (a->window > 0) keys = std::min<int64_t>(keys, a->window);
  const int64_t max_tiles = std::max<int64_t>(1, (keys + g4::kTileN - 1) / g4::kTileN);
  const int64_t units = std::max<int64_t>(1, int64_t(a->batch) * a->num_kv_heads);
  int64_t n = (sm_count() + units - 1) / units;
  n = std::max<int64_t>(1, std::min<int64_t>(std::min(n, max_tiles), g4::kDecodeMaxSplits));
  const int64_t tps = (max_tiles + n - 1) / n;
  return static_cast<int>((max_tiles + tps - 1) / tps);
}

// Upper bound of scratch tiles per query head for the materialised backward:
// exact band sizes for fixed layouts, a per-tile bound for packed layouts.
int64_t mat_head_cap_tiles(const g4_attn_args* a, int n_qt_total) {
  const bool packed = a->cu_seqlens_q != nullptr;
  const int W = a->window;
  if (packed) {
    const int64_t kmax = (a->max_seqlen_k + g4::kTileN - 1) / g4::kTileN;
    int64_t per = kmax;
    if (W > 0) per = std::min<int64_t>(per, (W + 126) / g4::kTileN + 2);
    return per * n_qt_total;
  }
  const int n_qt = (a->seqlen_q + g4::kTileM - 1) / g4::kTileM;
  const int q_off = a->seqlen_k - a->seqlen_q;
  int64_t total = 0;
  for (int qt = 0; qt < n_qt; ++qt) {
    const int qa0 = qt * g4::kTileM + q_off;
    const int qa1 = std::min((qt + 1) * g4::kTileM, a->seqlen_q) - 1 + q_off;
    const int lo = W > 0 ? std::max(0, qa0 - W + 1) : 0;
    const int hi = std::min(qa1, a->seqlen_k - 1);
    if (hi >= lo) total += hi / g4::kTileN - lo / g4::kTileN + 1;
  }
  return total * a->batch;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace modes: 0 single-kernel forward, 1 backward with recompute kernels,
// 2 backward with materialised P/dS tiles, 3 two-pass forward (d512, P tiles).
// Modes 2 and 3 fall back to 1 / 0 when the call is not eligible (vision
// metadata needs data-dependent key ranges; the two-pass forward is d512 only).
Workspace plan_workspace(const g4_attn_args* a, int mode) {
  Workspace w;
  const bool packed = a->cu_seqlens_q != nullptr;
  if ((mode == 0 || mode == 3) && decode_eligible(a)) {
    size_t off = 256;
    w.decode = true;
    w.decode_splits = decode_splits(a);
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
  if (a->vision_ids && a->window > 0) {
    const int64_t meta_len = packed ? a->seqlen_k : int64_t(a->batch) * a->seqlen_k;
    w.pair_last = off;
    off = align256(off + sizeof(int) * meta_len);
    if (backward) {
      w.pair_first = off;
      off = align256(off + sizeof(int) * meta_len);
    }
  }
  if (backward) {
    w.tokens_q = packed ? a->seqlen_q : int64_t(a->batch) * a->seqlen_q;
    w.delta = off;
    off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
    w.lse2 = off;
    off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
    if (backward == 2 && !(a->vision_ids && a->window > 0)) {
      w.materialized = true;
      w.n_qt_total = packed ? w.max_q_tiles
                            : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
      if (packed) {
        w.seg_first = off;
        off = align256(off + sizeof(int) * a->batch);
      }
      w.ranges = off;
      off = align256(off + sizeof(int4) * w.n_qt_total);
      w.head_cap_tiles = mat_head_cap_tiles(a, w.n_qt_total);
      const size_t tiles = size_t(a->num_q_heads) * size_t(w.head_cap_tiles) * 32768;
      w.p_tiles = off;
      off = align256(off + tiles);
      w.ds_tiles = off;
      off = align256(off + tiles);
    }
  }
  if (two_pass_fwd) {
    w.materialized = true;
    w.tokens_q = packed ? a->seqlen_q : int64_t(a->batch) * a->seqlen_q;
    w.n_qt_total = packed ? w.max_q_tiles
                          : a->batch * ((a->seqlen_q + g4::kTileM - 1) / g4::kTileM);
    w.ranges = off;
    off = align256(off + sizeof(int4) * w.n_qt_total);
    w.head_cap_tiles = mat_head_cap_tiles(a, w.n_qt_total);
    const size_t tiles = size_t(a->num_q_heads) * size_t(w.head_cap_tiles);
    w.p_tiles = off;
    off = align256(off + tiles * 32768);
    w.fwd_alpha = off;
    off = align256(off + tiles * 128 * sizeof(float));
    w.fwd_flags = off;
    off = align256(off + tiles * sizeof(int));
    w.fwd_inv_l = off;
    off = align256(off + sizeof(float) * a->num_q_heads * w.tokens_q);
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
  return l;
}

// Common prologue: zero the header, plan packed tiles and metadata bounds.
int prepare(const g4_attn_args* a, const Workspace& w, bool backward, cudaStream_t st,
            g4::MaskSpec* mask) {
  if (!a->workspace || a->workspace_bytes < w.total)
    return fail(G4_ERR_WORKSPACE, "workspace of %zu bytes required", w.total);
  cudaError_t e = cudaMemsetAsync(a->workspace, 0, 256, st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace reset");
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

// Single-token decode: split-key kernel, then the merge of the splits.
int run_decode(const g4_attn_args* a, cudaStream_t st) {
  const Workspace w = plan_workspace(a, 0);
  if (!a->workspace || a->workspace_bytes < w.total)
    return fail(G4_ERR_WORKSPACE, "workspace of %zu bytes required", w.total);
  cudaError_t ce = cudaMemsetAsync(a->workspace, 0, 256, st);
  if (ce != cudaSuccess) return cuda_fail(ce, "workspace reset");
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
  return plan_workspace(args, 3).total;
}

size_t g4_attn_fwd_min_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  return plan_workspace(args, 0).total;
}

size_t g4_attn_bwd_workspace_bytes(const g4_attn_args* args) {
  if (!args) return 0;
  return plan_workspace(args, 2).total;
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
  // Two-pass d512 forward (P tiles in HBM, no QK^T recomputation) when the
  // workspace holds its scratch; otherwise the single-kernel forward.
  const Workspace w3 = plan_workspace(a, 3);
  const Workspace w =
      (w3.materialized && a->workspace && a->workspace_bytes >= w3.total) ? w3 : plan_workspace(a, 0);
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
  if (w.materialized) {
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
    m.head_cap_tiles = w.head_cap_tiles;
    m.p_tiles = ws_ptr<uint8_t>(a, w.p_tiles);
    m.fwd_alpha = ws_ptr<float>(a, w.fwd_alpha);
    m.fwd_flags = ws_ptr<int>(a, w.fwd_flags);
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
    int e;
    {
      LaunchScope ls(kKPlan, st);
      e = g4::launch_plan_qtile_ranges(m, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "query-tile range planning");
    }
    {
      LaunchScope ls(kKFwdScore, st);
      e = g4::launch_bwd_score(D, 2, tq, tk, tv, tq, m, w.n_qt_total, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "forward score launch");
    }
    CUtensorMap to128;  // O, written by TMA stores in 128-row tiles
    if ((rc = make_map(&to128, a->o, a->head_dim_v, a->num_q_heads, a->seqlen_q, bq,
                       a->o_stride[2], a->o_stride[1], a->o_stride[0], 128)))
      return rc;
    {
      LaunchScope ls(kKFwdPv, st);
      CUtensorMap tp;  // the P scratch as bytes: the d512 O = P V GEMM runs as CTA pairs
      const bool pairs = g4::gemm_pairs_ok(D, 3, m);
      if (pairs && (rc = make_scratch_map(&tp, m.p_tiles,
                                          2 * int64_t(a->num_q_heads) * w.head_cap_tiles)))
        return rc;
      e = g4::launch_bwd_tile_gemm(D, 3, tv64, to128, pairs ? &tp : nullptr, m, w.n_qt_total,
                                   a->num_q_heads, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "forward PV launch");
    }
    return G4_OK;
  }
  const int slabs = a->head_dim_v / 256;
  LaunchScope ls(kKFwd, st);
  int e = D == 256 ? g4::launch_fwd<256>(tq, tk, tv, p, grid_x, a->num_q_heads, slabs, st)
                   : g4::launch_fwd<512>(tq, tk, tv, p, grid_x, a->num_q_heads, slabs, st);
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
  // Materialised P/dS when eligible and the workspace holds the scratch,
  // otherwise the recompute kernels (small workspaces, vision metadata).
  const Workspace wm = plan_workspace(a, 2);
  const Workspace w =
      (wm.materialized && a->workspace && a->workspace_bytes >= wm.total) ? wm : plan_workspace(a, 1);
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
    e = g4::launch_bwd_preprocess(p, a->head_dim_v, w.tokens_q, st);
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
  if (w.materialized) {
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
    m.head_cap_tiles = w.head_cap_tiles;
    m.p_tiles = ws_ptr<uint8_t>(a, w.p_tiles);
    m.ds_tiles = ws_ptr<uint8_t>(a, w.ds_tiles);
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
    CUtensorMap tq64, tdo64;
    if ((rc = make_map(&tq64, a->q, D, a->num_q_heads, a->seqlen_q, bq, a->q_stride[2],
                       a->q_stride[1], a->q_stride[0], 64)))
      return rc;
    if ((rc = make_map(&tdo64, a->dout, a->head_dim_v, a->num_q_heads, a->seqlen_q, bq,
                       a->do_stride[2], a->do_stride[1], a->do_stride[0], 64)))
      return rc;
    CUtensorMap tdq128, tdk128, tdv128;  // gradients, written by TMA stores in 128-row tiles
    if ((rc = make_map(&tdq128, a->dq, D, a->num_q_heads, a->seqlen_q, bq, a->dq_stride[2],
                       a->dq_stride[1], a->dq_stride[0], 128)))
      return rc;
    if ((rc = make_map(&tdk128, a->dk, D, a->num_kv_heads, a->seqlen_k, bq, a->dk_stride[2],
                       a->dk_stride[1], a->dk_stride[0], 128)))
      return rc;
    if ((rc = make_map(&tdv128, a->dv, a->head_dim_v, a->num_kv_heads, a->seqlen_k, bq,
                       a->dv_stride[2], a->dv_stride[1], a->dv_stride[0], 128)))
      return rc;
    {
      LaunchScope ls(kKPlan, st);
      e = g4::launch_plan_qtile_ranges(m, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "query-tile range planning");
    }
    for (int pass = 0; pass < (D == 512 ? 2 : 1); ++pass) {
      LaunchScope ls(kKScore, st);
      e = g4::launch_bwd_score(D, pass, tq, tk, tv, tdo, m, w.n_qt_total, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "score launch");
    }
    // dV and dK in one launch evens out the end of the KV-major grid, but it
    // streams both B operands (dO and Q) at once: only when together they take
    // at most 80 MiB of the 126 MB L2 (measured: 64 MiB, -12%; 256 MiB, no gain).
    const int64_t b_bytes =
        int64_t(w.tokens_q) * a->num_q_heads * (int64_t(D) + a->head_dim_v) * 2;
    if (b_bytes <= (int64_t(80) << 20)) {
      LaunchScope ls(kKGemmDvDk, st);
      e = g4::launch_bwd_tile_gemm_dvdk(D, tdo64, tdv128, tq64, tdk128, m, gk, a->num_kv_heads,
                                        st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "dV/dK launch");
    } else {
      {
        LaunchScope ls(kKGemmDv, st);
        e = g4::launch_bwd_tile_gemm(D, 0, tdo64, tdv128, nullptr, m, gk, a->num_kv_heads, st);
        if (e) return cuda_fail(static_cast<cudaError_t>(e), "dV launch");
      }
      LaunchScope ls(kKGemmDk, st);
      e = g4::launch_bwd_tile_gemm(D, 1, tq64, tdk128, nullptr, m, gk, a->num_kv_heads, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "dK launch");
    }
    {
      LaunchScope ls(kKGemmDq, st);
      CUtensorMap tds;  // the dS scratch as bytes: the d512 dQ GEMM runs as CTA pairs
      const bool pairs = g4::gemm_pairs_ok(D, 2, m);
      if (pairs && (rc = make_scratch_map(&tds, m.ds_tiles,
                                          2 * int64_t(a->num_q_heads) * w.head_cap_tiles)))
        return rc;
      e = g4::launch_bwd_tile_gemm(D, 2, tk64, tdq128, pairs ? &tds : nullptr, m, w.n_qt_total,
                                   a->num_q_heads, st);
      if (e) return cuda_fail(static_cast<cudaError_t>(e), "dQ launch");
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
