// extern "C" entry points of libps_b200.so (declared in include/ps_b200.h):
// argument validation, TMA descriptor encoding and kernel launches.
#include "ps_b200.h"
#include "internal.h"

#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>

namespace psb {

namespace {
thread_local char g_msg[512] = "";

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// The kernels are compiled for sm_100a only; refuse other devices up front.
int check_device() {
  static int verdict[64] = {0};  // 0 unknown, 1 ok, 2 unsupported
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev >= 0 && dev < 64 && verdict[dev] == 1) return PS_B200_OK;
  int major = 0, minor = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) return set_cuda_error("cudaDeviceGetAttribute", e);
  const bool ok = major == 10 && minor == 0;
  if (dev >= 0 && dev < 64) verdict[dev] = ok ? 1 : 2;
  if (!ok)
    return set_error(PS_B200_ERR_UNSUPPORTED, "libps_b200 is built for sm_100a; device %d is sm_%d%d", dev, major,
                     minor);
  return PS_B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
  if (dev >= 0 && dev < 64) cached[dev] = sms;
  return sms;
}

std::atomic<unsigned long long> g_launches{0};

bool is16bit(int dtype) { return dtype == PS_B200_BF16 || dtype == PS_B200_FP16; }

// 5-D map over [batch][seg][row][head][d] with a (64 x 1 x 128 x 1 x 1) box:
// one 64-column, 128-row half tile with 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, bool fp16, int head_dim, int heads, int seg_rows, int segs,
             int batch, const int64_t st[4]) {
  auto fn = encode_fn();
  if (!fn) return set_error(PS_B200_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  // Byte strides of the head, row, segment and batch axes.  Axes of extent 1
  // get the span of the axes below them so the map stays well formed.
  int64_t sh = st[3] * 2, sr = st[2] * 2, ss = st[1] * 2, sb = st[0] * 2;
  if (heads == 1) sh = int64_t(head_dim) * 2;
  if (seg_rows == 1) sr = sh * heads;
  if (segs == 1) ss = sr * seg_rows;
  if (batch == 1) sb = ss * segs;
  const int64_t strides_b[4] = {sh, sr, ss, sb};
  for (int i = 0; i < 4; ++i)
    if (strides_b[i] <= 0 || strides_b[i] % 16 != 0 || strides_b[i] >= (int64_t(1) << 40))
      return set_error(PS_B200_ERR_INVALID, "stride %lld bytes of axis %d is not a positive multiple of 16",
                       (long long)strides_b[i], 4 - i);
  cuuint64_t dims[5] = {cuuint64_t(head_dim), cuuint64_t(heads), cuuint64_t(seg_rows), cuuint64_t(segs),
                        cuuint64_t(batch)};
  cuuint64_t strides[4] = {cuuint64_t(sh), cuuint64_t(sr), cuuint64_t(ss), cuuint64_t(sb)};
  cuuint32_t box[5] = {64, 1, 128, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PS_B200_ERR_INVALID, "cuTensorMapEncodeTiled failed with CUresult %d", int(r));
  return PS_B200_OK;
}

// An explicit per-segment row table must have world entries in [0, seg_rows]
// summing to total.
int check_seg_valid(const int* seg_valid, int world, int seg_rows, int total) {
  if (!seg_valid) return PS_B200_OK;
  if (world > kMaxSegs) return set_error(PS_B200_ERR_UNSUPPORTED, "more than %d segments", kMaxSegs);
  int64_t sum = 0;
  for (int s = 0; s < world; ++s) {
    if (seg_valid[s] < 0 || seg_valid[s] > seg_rows)
      return set_error(PS_B200_ERR_INVALID, "segment %d holds %d rows, outside [0, %d]", s, seg_valid[s], seg_rows);
    sum += seg_valid[s];
  }
  if (sum != total) return set_error(PS_B200_ERR_INVALID, "segment rows sum to %lld, not total %d", (long long)sum, total);
  return PS_B200_OK;
}

// Valid rows per segment when `len` rows fill segments of `seg_rows` in order
// (ceil-width token shards: only the last non-empty segment is short).
void fill_valid(int* valid, int segs, int seg_rows, int len) {
  for (int s = 0; s < segs; ++s) {
    const int64_t v = int64_t(len) - int64_t(s) * seg_rows;
    valid[s] = int(v < 0 ? 0 : (v > seg_rows ? seg_rows : v));
  }
}

struct SegTensor {
  const void* ptr;
  int64_t st[4];
  int heads;  // extent of the head axis in the map
};

// Optional prefix range (joint attention): queries/keys [0, len) from its own
// tensors, ahead of the segmented range.
struct Prefix {
  SegTensor q, k, v;
  void* out = nullptr;
  int64_t out_st[4] = {0, 0, 0, 0};
  int len = 0;
};

int attention_common(const SegTensor& q, const SegTensor& k, const SegTensor& v, void* out,
                     const int64_t out_st[4], int dtype, int out_dtype, int batch, int grid_heads, int group,
                     int head_dim,
                     int seg_rows_q, int segs_q, int len_q, int seg_rows_k, int segs_k, int len_k,
                     float softmax_scale, void* workspace, size_t workspace_bytes, int* status, void* stream,
                     const Prefix* pre = nullptr, const int* seg_valid = nullptr, void* const* seg_out = nullptr) {
  const int pre_len = pre ? pre->len : 0;
  if (segs_q > kMaxSegs || segs_k > kMaxSegs)
    return set_error(PS_B200_ERR_UNSUPPORTED, "more than %d segments", kMaxSegs);
  if (!is16bit(dtype)) return set_error(PS_B200_ERR_UNSUPPORTED, "attention supports bf16 and fp16 only");
  if (out_dtype != dtype && out_dtype != PS_B200_FP32)
    return set_error(PS_B200_ERR_UNSUPPORTED, "attention output must be fp32 or the input dtype");
  if (head_dim != 128) return set_error(PS_B200_ERR_UNSUPPORTED, "attention supports head_dim 128 only (got %d)", head_dim);
  if (batch < 0 || grid_heads < 0 || len_q < 0 || len_k < 0 || group < 1)
    return set_error(PS_B200_ERR_INVALID, "negative size");
  if (pre_len < 0) return set_error(PS_B200_ERR_INVALID, "negative prefix length");
  if (batch == 0 || grid_heads == 0 || len_q + pre_len == 0) return PS_B200_OK;
  if (len_k + pre_len == 0) return set_error(PS_B200_ERR_INVALID, "empty key set");
  if (seg_rows_q <= 0 || segs_q <= 0 || seg_rows_k <= 0 || segs_k <= 0)
    return set_error(PS_B200_ERR_INVALID, "segment geometry must be positive");
  if (int64_t(seg_rows_q) * segs_q < len_q || int64_t(seg_rows_k) * segs_k < len_k)
    return set_error(PS_B200_ERR_INVALID, "len exceeds segments * seg_rows");
  if (batch > 65535 || grid_heads > 65535) return set_error(PS_B200_ERR_UNSUPPORTED, "batch/heads above 65535");
  if (!std::isfinite(softmax_scale)) return set_error(PS_B200_ERR_INVALID, "softmax_scale must be finite");
  if (!q.ptr || !k.ptr || !v.ptr || (!out && !seg_out)) return set_error(PS_B200_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q.ptr) || !aligned16(k.ptr) || !aligned16(v.ptr) || !aligned16(out))
    return set_error(PS_B200_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if (seg_out)
    for (int s = 0; s < segs_q; ++s)
      if (!seg_out[s] || !aligned16(seg_out[s]))
        return set_error(PS_B200_ERR_INVALID, "segment %d output pointer null or not 16-byte aligned", s);
  if (pre_len) {
    if (!pre->q.ptr || !pre->k.ptr || !pre->v.ptr || !pre->out)
      return set_error(PS_B200_ERR_INVALID, "null prefix tensor pointer");
    if (!aligned16(pre->q.ptr) || !aligned16(pre->k.ptr) || !aligned16(pre->v.ptr) || !aligned16(pre->out))
      return set_error(PS_B200_ERR_INVALID, "prefix tensor pointers must be 16-byte aligned");
    for (int i = 0; i < 4; ++i)
      if (pre->out_st[i] < 0 || pre->out_st[i] % 8 != 0)
        return set_error(PS_B200_ERR_INVALID, "prefix output strides must be non-negative multiples of 8");
  }
  for (int i = 0; i < 4; ++i)
    if (out_st[i] < 0 || out_st[i] % 8 != 0)
      return set_error(PS_B200_ERR_INVALID, "output strides must be non-negative multiples of 8 elements");
  if (status && (reinterpret_cast<uintptr_t>(status) & 3u) != 0)
    return set_error(PS_B200_ERR_INVALID, "status word must be 4-byte aligned");
  if (int rc = check_device()) return rc;
  const bool fp16 = dtype == PS_B200_FP16;
  CUtensorMap tq, tk, tv;
  if (int rc = make_map(&tq, q.ptr, fp16, head_dim, q.heads, seg_rows_q, segs_q, batch, q.st)) return rc;
  if (int rc = make_map(&tk, k.ptr, fp16, head_dim, k.heads, seg_rows_k, segs_k, batch, k.st)) return rc;
  if (int rc = make_map(&tv, v.ptr, fp16, head_dim, v.heads, seg_rows_k, segs_k, batch, v.st)) return rc;
  CUtensorMap tqp = tq, tkp = tk, tvp = tv;
  if (pre_len) {
    if (int rc = make_map(&tqp, pre->q.ptr, fp16, head_dim, pre->q.heads, pre_len, 1, batch, pre->q.st)) return rc;
    if (int rc = make_map(&tkp, pre->k.ptr, fp16, head_dim, pre->k.heads, pre_len, 1, batch, pre->k.st)) return rc;
    if (int rc = make_map(&tvp, pre->v.ptr, fp16, head_dim, pre->v.heads, pre_len, 1, batch, pre->v.st)) return rc;
  }
  AttnArgs a{};
  const int64_t osize = out_dtype == PS_B200_FP32 ? 4 : 2;
  for (int s = 0; s < segs_q; ++s)
    a.seg_out[s] = seg_out ? seg_out[s] : static_cast<void*>(static_cast<char*>(out) + s * out_st[1] * osize);
  for (int i = 0; i < 4; ++i) a.o_stride[i] = out_st[i];
  a.seg_rows_q = seg_rows_q;
  a.nsegs_q = segs_q;
  a.q_tiles_per_seg = (seg_rows_q + 127) / 128;
  a.seg_rows_k = seg_rows_k;
  a.nsegs_k = segs_k;
  if (seg_valid) {  // explicit per-segment rows (queries and keys share the segments)
    for (int s = 0; s < segs_q; ++s) {
      if (seg_valid[s] < 0 || seg_valid[s] > seg_rows_q)
        return set_error(PS_B200_ERR_INVALID, "segment %d valid rows %d outside [0, %d]", s, seg_valid[s], seg_rows_q);
      a.valid_q[s] = a.valid_k[s] = seg_valid[s];
    }
  } else {
    fill_valid(a.valid_q, segs_q, seg_rows_q, len_q);
    fill_valid(a.valid_k, segs_k, seg_rows_k, len_k);
  }
  // Query tiles are laid out segment-major (tiles past a segment's valid rows
  // compute on padding and store nothing); trailing empty segments are dropped.
  int last_q = segs_q - 1;
  while (last_q >= 0 && a.valid_q[last_q] == 0) --last_q;
  a.num_q_tiles = (last_q + 1) * a.q_tiles_per_seg;
  a.num_kv_tiles = 0;
  for (int s = 0; s < segs_k; ++s) a.num_kv_tiles += (a.valid_k[s] + 127) / 128;
  a.group = group;
  a.scale_log2 = static_cast<float>(double(softmax_scale) * 1.4426950408889634);
  a.out_fp32 = out_dtype == PS_B200_FP32;
  a.status = status;
  a.pre_len = pre_len;
  a.pre_tiles = (pre_len + 127) / 128;
  a.num_q_tiles += a.pre_tiles;
  a.num_kv_tiles += a.pre_tiles;
  a.pre_out = pre_len ? pre->out : out;
  for (int i = 0; i < 4; ++i) a.pre_o_stride[i] = pre_len ? pre->out_st[i] : out_st[i];
  // Work units (tile pair, head, batch).  The last, partial wave's units are
  // split along the key range when a workspace is given, so that wave ends
  // about `split` times sooner.
  a.npairs = (a.num_q_tiles + 1) / 2;
  a.grid_heads = grid_heads;
  const int64_t units = int64_t(a.npairs) * grid_heads * batch;
  a.full_units = static_cast<int>(units < 0x7fffffff ? units : 0x7fffffff);
  a.split = 1;
  if (workspace && workspace_bytes >= size_t(kAttnWorkspaceBytes) && aligned16(workspace)) {
    const int sms = sm_count();
    const int64_t rem = units % sms;
    if (rem > 0 && sms <= 160) {
      int split = static_cast<int>(sms / rem);
      split = split < kMaxSplit ? split : kMaxSplit;
      split = split < a.num_kv_tiles / 2 ? split : a.num_kv_tiles / 2;  // at least two key tiles per part
      if (split >= 2) {
        a.split = split;
        a.full_units = static_cast<int>(units - rem);
        a.ws_o = static_cast<float*>(workspace);
        a.ws_lse = a.ws_o + rem * split * 2 * 128 * 128;
      }
    }
  }
  return launch_attention(tq, tk, tv, tqp, tkp, tvp, a, units, fp16, static_cast<cudaStream_t>(stream));
}

}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t err) {
  return set_error(PS_B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace psb

using namespace psb;

// Shared body of ps_b200_prepass / ps_b200_prepass_to: dst[d] is the
// [3][seg_rows][heads_per_rank][head_dim] block for destination rank d.
static int prepass_common(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                   const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                   const float* freqs, int64_t freqs_row_stride, void* const* dst, int dtype,
                   int world, int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, float eps,
                   int norm_rope, int rope_style, int rope_pairs, void* stream, void* q_out = nullptr,
                   int kv_fanout = 0, int batch = 1, const int64_t* x_batch_strides = nullptr,
                   int64_t freqs_batch_stride = 0) {
  if (!is16bit(dtype)) return set_error(PS_B200_ERR_UNSUPPORTED, "prepass supports bf16 and fp16 only");
  if (batch < 0 || batch > 65535) return set_error(PS_B200_ERR_INVALID, "batch must be in [0, 65535]");
  if (batch == 0) return PS_B200_OK;
  if (batch > 1) {
    if (!x_batch_strides) return set_error(PS_B200_ERR_INVALID, "batch > 1 needs x_batch_strides");
    for (int i = 0; i < 3; ++i)
      if (x_batch_strides[i] < 0 || x_batch_strides[i] % 8 != 0)
        return set_error(PS_B200_ERR_INVALID, "x_batch_strides must be non-negative multiples of 8");
    if (freqs_batch_stride < 0 || freqs_batch_stride % 4 != 0)
      return set_error(PS_B200_ERR_INVALID, "freqs_batch_stride must be a non-negative multiple of 4");
  }
  if (world < 1 || n_local < 0 || seg_rows < n_local || heads < 1 || heads_per_rank < 1 ||
      int64_t(heads_per_rank) * world < heads || head_dim <= 0)
    return set_error(PS_B200_ERR_INVALID, "inconsistent prepass geometry");
  if (head_dim % 8 != 0) return set_error(PS_B200_ERR_UNSUPPORTED, "head_dim must be a multiple of 8");
  if (norm_rope < 0 || norm_rope > 2) return set_error(PS_B200_ERR_INVALID, "norm_rope must be 0, 1 or 2");
  if (norm_rope == 2 && (head_dim / 8 > 32 || ((head_dim / 8) & (head_dim / 8 - 1)) != 0))
    return set_error(PS_B200_ERR_UNSUPPORTED, "per-head norm needs head_dim/8 a power of two <= 32");
  if (rope_style != 0 && rope_style != 1) return set_error(PS_B200_ERR_INVALID, "rope_style must be 0 or 1");
  if (norm_rope && rope_style == 0 && rope_pairs != head_dim / 2)
    return set_error(PS_B200_ERR_INVALID, "interleaved RoPE rotates head_dim/2 pairs (got %d)", rope_pairs);
  if (norm_rope && rope_style == 1) {
    if (rope_pairs <= 0 || rope_pairs % 8 != 0 || 2 * rope_pairs > head_dim)
      return set_error(PS_B200_ERR_UNSUPPORTED, "split-half RoPE needs rope_pairs a positive multiple of 8, "
                                                "2*rope_pairs <= head_dim (got %d)", rope_pairs);
    if (head_dim / 8 > 32 || ((head_dim / 8) & (head_dim / 8 - 1)) != 0)
      return set_error(PS_B200_ERR_UNSUPPORTED, "split-half RoPE needs head_dim/8 a power of two <= 32");
  }
  if (int64_t(heads) * head_dim > 8192)
    return set_error(PS_B200_ERR_UNSUPPORTED, "heads*head_dim above 8192 is not supported");
  if (seg_rows == 0) return PS_B200_OK;
  if (n_local > 0) {
    const void* xs[3] = {x_q, x_k, x_v};
    for (int i = 0; i < 3; ++i)
      if (!xs[i] || !aligned16(xs[i]) || !x_row_strides || x_row_strides[i] % 8 != 0 || x_row_strides[i] < 0 ||
          (x_head_strides && (x_head_strides[i] % 8 != 0 || x_head_strides[i] < 0)))
        return set_error(PS_B200_ERR_INVALID,
                         "projection inputs must be 16-byte aligned with row and head strides %% 8 == 0");
    if (norm_rope) {
      if (!w_qnorm || !w_knorm || !aligned16(w_qnorm) || !aligned16(w_knorm))
        return set_error(PS_B200_ERR_INVALID, "norm weights null or not 16-byte aligned");
      if (w_dtype != dtype && w_dtype != PS_B200_FP32)
        return set_error(PS_B200_ERR_UNSUPPORTED, "norm weights must be fp32 or the input dtype");
      if (!freqs || !aligned16(freqs) || freqs_row_stride % 4 != 0 || freqs_row_stride < 0)
        return set_error(PS_B200_ERR_INVALID, "freqs must be 16-byte aligned with a row stride %% 4 == 0");
      if (!std::isfinite(eps) || eps < 0.f) return set_error(PS_B200_ERR_INVALID, "eps must be finite and >= 0");
    }
  }
  if (int rc = check_device()) return rc;
  PrepassArgs a{};
  a.x[0] = x_q;
  a.x[1] = x_k;
  a.x[2] = x_v;
  for (int i = 0; i < 3; ++i) {
    a.x_batch_stride[i] = (batch > 1 && x_batch_strides) ? x_batch_strides[i] : 0;
    a.x_row_stride[i] = x_row_strides ? x_row_strides[i] : 0;
    a.x_head_stride[i] = x_head_strides ? x_head_strides[i] : head_dim;
  }
  a.freqs_batch_stride = batch > 1 ? freqs_batch_stride : 0;
  a.batch = batch;
  a.w[0] = w_qnorm;
  a.w[1] = w_knorm;
  a.w_fp32 = w_dtype == PS_B200_FP32;
  a.freqs = freqs;
  a.freqs_row_stride = freqs_row_stride;
  for (int d = 0; d < (kv_fanout > world ? kv_fanout : world); ++d) a.dst[d] = dst[d];
  a.q_out = q_out;
  a.kv_fanout = kv_fanout;
  a.world = world;
  a.n_local = n_local;
  a.seg_rows = seg_rows;
  a.heads = heads;
  a.heads_per_rank = heads_per_rank;
  a.head_dim = head_dim;
  a.eps = eps;
  a.norm_rope = norm_rope;
  a.rope_style = rope_style;
  a.rope_pairs = rope_pairs;
  return launch_prepass(a, dtype == PS_B200_FP16, static_cast<cudaStream_t>(stream));
}


// Shared body of the joint (prefix + segmented) Ulysses attention entries:
// image outputs go to out_send ([world][seg_rows][h][D]) or, with out_blocks,
// to one pointer per source segment (row stride out_row_stride).
static int joint_common(const void* recv, const void* prefix_qkv, void* out_send, void* const* out_blocks,
                        int64_t out_row_stride, void* prefix_out, int dtype, int out_dtype, int world, int seg_rows,
                        int total, int prefix_len, const int* seg_valid, int heads_per_rank, int heads_valid,
                        int head_dim, float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                        void* stream) {
  if (world < 1 || seg_rows < 1 || total < 1 || prefix_len < 0 || heads_per_rank < 1 || heads_valid < 0 ||
      heads_valid > heads_per_rank || int64_t(seg_rows) * world < total)
    return set_error(PS_B200_ERR_INVALID, "inconsistent joint Ulysses geometry");
  if (int rc = check_seg_valid(seg_valid, world, seg_rows, total)) return rc;
  if (heads_valid == 0) return PS_B200_OK;
  const int64_t D = head_dim, h = heads_per_rank, n = seg_rows, P = prefix_len;
  const int64_t block = n * h * D;
  const char* base = static_cast<const char*>(recv);
  const int64_t in_st[4] = {int64_t(world) * 3 * block, 3 * block, h * D, D};
  int64_t out_st[4] = {int64_t(world) * block, block, h * D, D};
  if (out_blocks) {
    out_st[0] = out_st[1] = 0;
    out_st[2] = out_row_stride;
  }
  SegTensor tq{base, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tk{base + block * 2, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tv{base + block * 4, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  Prefix pre;
  pre.len = prefix_len;
  if (prefix_len) {
    const char* pb = static_cast<const char*>(prefix_qkv);
    const int64_t pblock = P * h * D;
    const int64_t pst[4] = {3 * pblock, 3 * pblock, h * D, D};
    pre.q = SegTensor{pb, {pst[0], pst[1], pst[2], pst[3]}, heads_per_rank};
    pre.k = SegTensor{pb + pblock * 2, {pst[0], pst[1], pst[2], pst[3]}, heads_per_rank};
    pre.v = SegTensor{pb + pblock * 4, {pst[0], pst[1], pst[2], pst[3]}, heads_per_rank};
    pre.out = prefix_out;
    pre.out_st[0] = pblock;
    pre.out_st[1] = pblock;
    pre.out_st[2] = h * D;
    pre.out_st[3] = D;
  }
  return attention_common(tq, tk, tv, out_send, out_st, dtype, out_dtype, 1, heads_valid, 1, head_dim, seg_rows,
                          world, total, seg_rows, world, total, softmax_scale, workspace, workspace_bytes, status,
                          stream, &pre, seg_valid, out_blocks);
}

extern "C" {

int ps_b200_abi_version(void) { return PS_B200_ABI_VERSION; }

const char* ps_b200_last_error(void) { return psb::g_msg; }

int ps_b200_prepass(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                    const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                    const float* freqs, int64_t freqs_row_stride, void* send, int dtype, int world, int n_local,
                    int seg_rows, int heads, int heads_per_rank, int head_dim, float eps, int norm_rope,
                    int rope_style, int rope_pairs, void* stream) {
  if (world < 1 || world > kMaxSegs) return set_error(PS_B200_ERR_INVALID, "world must be in [1, %d]", kMaxSegs);
  if (!send || !aligned16(send)) {
    if (seg_rows > 0) return set_error(PS_B200_ERR_INVALID, "send buffer null or not 16-byte aligned");
  }
  void* dst[kMaxSegs];
  const int64_t block = int64_t(3) * seg_rows * heads_per_rank * head_dim * 2;  // bytes of one destination block
  for (int d = 0; d < world; ++d) dst[d] = static_cast<char*>(send) + d * block;
  return prepass_common(x_q, x_k, x_v, x_row_strides, x_head_strides, w_qnorm, w_knorm, w_dtype, freqs,
                        freqs_row_stride, dst, dtype, world, n_local, seg_rows, heads, heads_per_rank, head_dim,
                        eps, norm_rope, rope_style, rope_pairs, stream);
}

int ps_b200_prepass_to(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                       const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                       const float* freqs, int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int world,
                       int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, float eps,
                       int norm_rope, int rope_style, int rope_pairs, void* stream) {
  if (world < 1 || world > kMaxSegs) return set_error(PS_B200_ERR_INVALID, "world must be in [1, %d]", kMaxSegs);
  if (seg_rows > 0) {
    if (!dst_blocks) return set_error(PS_B200_ERR_INVALID, "null destination table");
    for (int d = 0; d < world; ++d)
      if (!dst_blocks[d] || !aligned16(dst_blocks[d]))
        return set_error(PS_B200_ERR_INVALID, "destination block %d null or not 16-byte aligned", d);
  }
  return prepass_common(x_q, x_k, x_v, x_row_strides, x_head_strides, w_qnorm, w_knorm, w_dtype, freqs,
                        freqs_row_stride, dst_blocks, dtype, world, n_local, seg_rows, heads, heads_per_rank,
                        head_dim, eps, norm_rope, rope_style, rope_pairs, stream);
}

int ps_b200_attn_fwd(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                     const void* v, const int64_t v_strides[4], void* out, const int64_t out_strides[4],
                     int dtype, int out_dtype, int batch, int heads_q, int heads_kv, int head_dim, int seg_rows_q,
                     int segs_q, int len_q, int seg_rows_k, int segs_k, int len_k, float softmax_scale,
                     void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (!q_strides || !k_strides || !v_strides || !out_strides) return set_error(PS_B200_ERR_INVALID, "null strides");
  if (heads_kv <= 0 || heads_q < 0 || heads_q % heads_kv != 0)
    return set_error(PS_B200_ERR_INVALID, "heads_q must be a positive multiple of heads_kv");
  SegTensor tq{q, {q_strides[0], q_strides[1], q_strides[2], q_strides[3]}, heads_q};
  SegTensor tk{k, {k_strides[0], k_strides[1], k_strides[2], k_strides[3]}, heads_kv};
  SegTensor tv{v, {v_strides[0], v_strides[1], v_strides[2], v_strides[3]}, heads_kv};
  return attention_common(tq, tk, tv, out, out_strides, dtype, out_dtype, batch, heads_q, heads_q / heads_kv, head_dim,
                          seg_rows_q, segs_q, len_q, seg_rows_k, segs_k, len_k, softmax_scale, workspace,
                          workspace_bytes, status, stream);
}

int ps_b200_prepass_token_to(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                             const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                             const float* freqs, int64_t freqs_row_stride, void* q_out, void* const* kv_dst,
                             int ndst, int dtype, int n_local, int width, int heads, int head_dim, float eps,
                             int norm_rope, int rope_style, int rope_pairs, void* stream) {
  if (ndst < 1 || ndst > kMaxSegs) return set_error(PS_B200_ERR_INVALID, "1..%d k/v destinations", kMaxSegs);
  if (width > 0) {
    if (!q_out || !aligned16(q_out)) return set_error(PS_B200_ERR_INVALID, "q output null or not 16-byte aligned");
    if (!kv_dst) return set_error(PS_B200_ERR_INVALID, "null k/v destination table");
    for (int d = 0; d < ndst; ++d)
      if (!kv_dst[d] || !aligned16(kv_dst[d]))
        return set_error(PS_B200_ERR_INVALID, "k/v destination %d null or not 16-byte aligned", d);
  }
  return prepass_common(x_q, x_k, x_v, x_row_strides, x_head_strides, w_qnorm, w_knorm, w_dtype, freqs,
                        freqs_row_stride, kv_dst, dtype, 1, n_local, width, heads, heads, head_dim, eps, norm_rope,
                        rope_style, rope_pairs, stream, q_out, ndst);
}

int ps_b200_ulysses_attn_fwd(const void* recv, void* out_send, int dtype, int out_dtype, int world, int seg_rows,
                             int total, const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                             float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                             void* stream) {
  if (world < 1 || seg_rows < 0 || total < 0 || heads_per_rank < 1 || heads_valid < 0 ||
      heads_valid > heads_per_rank || int64_t(seg_rows) * world < total)
    return set_error(PS_B200_ERR_INVALID, "inconsistent Ulysses geometry");
  if (int rc = check_seg_valid(seg_valid, world, seg_rows, total)) return rc;
  if (total == 0 || heads_valid == 0) return PS_B200_OK;
  const int64_t D = head_dim, h = heads_per_rank, n = seg_rows;
  const int64_t block = n * h * D;  // one [seg_rows][h][D] block
  const char* base = static_cast<const char*>(recv);
  const int64_t in_st[4] = {int64_t(world) * 3 * block, 3 * block, h * D, D};
  const int64_t out_st[4] = {int64_t(world) * block, block, h * D, D};  // elements of out_dtype
  SegTensor tq{base, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tk{base + block * 2, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tv{base + block * 4, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  return attention_common(tq, tk, tv, out_send, out_st, dtype, out_dtype, 1, heads_valid, 1, head_dim, seg_rows, world, total,
                          seg_rows, world, total, softmax_scale, workspace, workspace_bytes, status, stream, nullptr,
                          seg_valid);
}

int ps_b200_ulysses_attn_to(const void* recv, void* const* out_blocks, int64_t out_row_stride, int dtype,
                            int out_dtype, int world, int seg_rows, int total, const int* seg_valid,
                            int heads_per_rank, int heads_valid, int head_dim, float softmax_scale, void* workspace,
                            size_t workspace_bytes, int* status, void* stream) {
  return ps_b200_ulysses_attn_batch(recv, out_blocks, 0, out_row_stride, dtype, out_dtype, 1, world, seg_rows,
                                    total, seg_valid, heads_per_rank, heads_valid, head_dim, softmax_scale,
                                    workspace, workspace_bytes, status, stream);
}

int ps_b200_ulysses_attn_batch(const void* recv, void* const* out_blocks, int64_t out_batch_stride,
                               int64_t out_row_stride, int dtype, int out_dtype, int batch, int world, int seg_rows,
                               int total, const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                               float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                               void* stream) {
  if (world < 1 || seg_rows < 0 || total < 0 || heads_per_rank < 1 || heads_valid < 0 ||
      heads_valid > heads_per_rank || int64_t(seg_rows) * world < total || batch < 0)
    return set_error(PS_B200_ERR_INVALID, "inconsistent Ulysses geometry");
  if (int rc = check_seg_valid(seg_valid, world, seg_rows, total)) return rc;
  if (total == 0 || heads_valid == 0 || batch == 0) return PS_B200_OK;
  if (!out_blocks) return set_error(PS_B200_ERR_INVALID, "null output table");
  if (out_row_stride < int64_t(heads_valid) * head_dim)
    return set_error(PS_B200_ERR_INVALID, "output row stride below heads_valid * head_dim");
  if (batch > 1 && out_batch_stride < 0) return set_error(PS_B200_ERR_INVALID, "negative output batch stride");
  const int64_t D = head_dim, h = heads_per_rank, n = seg_rows, B = batch;
  const int64_t block = n * h * D;  // one [seg_rows][h][D] block of one batch row
  const char* base = static_cast<const char*>(recv);
  // recv [world][3][batch][seg_rows][h][D]: strides {batch, segment, row, head}
  const int64_t in_st[4] = {block, 3 * B * block, h * D, D};
  const int64_t out_st[4] = {batch > 1 ? out_batch_stride : 0, 0, out_row_stride, D};
  SegTensor tq{base, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tk{base + B * block * 2, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  SegTensor tv{base + B * block * 4, {in_st[0], in_st[1], in_st[2], in_st[3]}, heads_per_rank};
  return attention_common(tq, tk, tv, nullptr, out_st, dtype, out_dtype, batch, heads_valid, 1, head_dim, seg_rows,
                          world, total, seg_rows, world, total, softmax_scale, workspace, workspace_bytes, status,
                          stream, nullptr, seg_valid, out_blocks);
}

int ps_b200_prepass_batch(const void* x_q, const void* x_k, const void* x_v, const int64_t x_batch_strides[3],
                          const int64_t x_row_strides[3], const int64_t x_head_strides[3], const void* w_qnorm,
                          const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_batch_stride,
                          int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int batch, int world,
                          int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, float eps,
                          int norm_rope, int rope_style, int rope_pairs, void* stream) {
  if (world < 1 || world > kMaxSegs) return set_error(PS_B200_ERR_INVALID, "world must be in [1, %d]", kMaxSegs);
  if (seg_rows > 0 && batch > 0) {
    if (!dst_blocks) return set_error(PS_B200_ERR_INVALID, "null destination table");
    for (int d = 0; d < world; ++d)
      if (!dst_blocks[d] || !aligned16(dst_blocks[d]))
        return set_error(PS_B200_ERR_INVALID, "destination block %d null or not 16-byte aligned", d);
  }
  return prepass_common(x_q, x_k, x_v, x_row_strides, x_head_strides, w_qnorm, w_knorm, w_dtype, freqs,
                        freqs_row_stride, dst_blocks, dtype, world, n_local, seg_rows, heads, heads_per_rank,
                        head_dim, eps, norm_rope, rope_style, rope_pairs, stream, nullptr, 0, batch,
                        x_batch_strides, freqs_batch_stride);
}

int ps_b200_ulysses_joint_attn_fwd(const void* recv, const void* prefix_qkv, void* out_send, void* prefix_out,
                                   int dtype, int out_dtype, int world, int seg_rows, int total, int prefix_len,
                                   const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                                   float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                                   void* stream) {
  return joint_common(recv, prefix_qkv, out_send, nullptr, 0, prefix_out, dtype, out_dtype, world, seg_rows, total,
                      prefix_len, seg_valid, heads_per_rank, heads_valid, head_dim, softmax_scale, workspace,
                      workspace_bytes, status, stream);
}

int ps_b200_ulysses_joint_attn_to(const void* recv, const void* prefix_qkv, void* const* out_blocks,
                                  int64_t out_row_stride, void* prefix_out, int dtype, int out_dtype, int world,
                                  int seg_rows, int total, int prefix_len, const int* seg_valid, int heads_per_rank,
                                  int heads_valid, int head_dim, float softmax_scale, void* workspace,
                                  size_t workspace_bytes, int* status, void* stream) {
  if (!out_blocks) return set_error(PS_B200_ERR_INVALID, "null output table");
  if (out_row_stride < int64_t(heads_valid) * head_dim)
    return set_error(PS_B200_ERR_INVALID, "output row stride below heads_valid * head_dim");
  return joint_common(recv, prefix_qkv, nullptr, out_blocks, out_row_stride, prefix_out, dtype, out_dtype, world,
                      seg_rows, total, prefix_len, seg_valid, heads_per_rank, heads_valid, head_dim, softmax_scale,
                      workspace, workspace_bytes, status, stream);
}

int ps_b200_broadcast(void* const* dst, int ndst, const void* src, size_t bytes, void* stream) {
  if (ndst < 1 || ndst > kMaxSegs) return set_error(PS_B200_ERR_INVALID, "1..%d destinations", kMaxSegs);
  if (bytes == 0) return PS_B200_OK;
  if (!src || !dst || !aligned16(src) || bytes % 16 != 0)
    return set_error(PS_B200_ERR_INVALID, "broadcast: 16-byte aligned source and a multiple of 16 bytes");
  for (int d = 0; d < ndst; ++d)
    if (!dst[d] || !aligned16(dst[d])) return set_error(PS_B200_ERR_INVALID, "broadcast destination %d", d);
  if (int rc = check_device()) return rc;
  BroadcastArgs a{};
  a.src = src;
  a.ndst = ndst;
  for (int d = 0; d < ndst; ++d) a.dst[d] = dst[d];
  a.vectors = static_cast<int64_t>(bytes / 16);
  return launch_broadcast(a, static_cast<cudaStream_t>(stream));
}

int ps_b200_unpack(const void* recv, void* out, int64_t out_row_stride, int dtype, int out_dtype, int world,
                   int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, void* stream) {
  if (world < 1 || n_local > seg_rows || heads_per_rank < 1 || int64_t(heads_per_rank) * world < heads)
    return set_error(PS_B200_ERR_INVALID, "inconsistent unpack geometry");
  return ps_b200_unpack_strided(recv, int64_t(seg_rows) * heads_per_rank * head_dim,
                                int64_t(heads_per_rank) * head_dim, out, out_row_stride, dtype, out_dtype, n_local,
                                heads, heads_per_rank, head_dim, stream);
}

int ps_b200_unpack_strided(const void* recv, int64_t src_stride, int64_t row_stride, void* out,
                           int64_t out_row_stride, int dtype, int out_dtype, int n_local, int heads,
                           int heads_per_rank, int head_dim, void* stream) {
  return ps_b200_unpack_batch(recv, src_stride, 0, row_stride, out, 0, out_row_stride, dtype, out_dtype, 1,
                              n_local, heads, heads_per_rank, head_dim, stream);
}

int ps_b200_unpack_batch(const void* recv, int64_t src_stride, int64_t batch_stride, int64_t row_stride, void* out,
                         int64_t out_batch_stride, int64_t out_row_stride, int dtype, int out_dtype, int batch,
                         int n_local, int heads, int heads_per_rank, int head_dim, void* stream) {
  if (!is16bit(dtype)) return set_error(PS_B200_ERR_UNSUPPORTED, "unpack supports bf16 and fp16 inputs only");
  if (out_dtype != dtype && out_dtype != PS_B200_FP32)
    return set_error(PS_B200_ERR_UNSUPPORTED, "unpack output must be fp32 or the input dtype");
  if (n_local < 0 || batch < 0 || heads < 1 || heads_per_rank < 1 || head_dim <= 0 || head_dim % 8 != 0)
    return set_error(PS_B200_ERR_INVALID, "inconsistent unpack geometry");
  if (int64_t(batch) * n_local * heads * (head_dim / 8) >= (int64_t(1) << 31))
    return set_error(PS_B200_ERR_UNSUPPORTED, "unpack size above 2^31 vectors");
  if (n_local == 0 || batch == 0) return PS_B200_OK;
  if (!recv || !out || !aligned16(recv) || !aligned16(out) || out_row_stride % 8 != 0 || out_row_stride < 0 ||
      src_stride % 8 != 0 || src_stride < 0 || row_stride % 8 != 0 || row_stride < 0 ||
      (batch > 1 && (batch_stride % 8 != 0 || batch_stride < 0 || out_batch_stride % 8 != 0 ||
                     out_batch_stride < 0)))
    return set_error(PS_B200_ERR_INVALID, "unpack buffers must be 16-byte aligned, strides %% 8 == 0");
  if (int rc = check_device()) return rc;
  UnpackArgs a{};
  a.recv = recv;
  a.src_stride = src_stride;
  a.batch_stride = batch > 1 ? batch_stride : 0;
  a.row_stride = row_stride;
  a.out = out;
  a.out_batch_stride = batch > 1 ? out_batch_stride : 0;
  a.out_row_stride = out_row_stride;
  a.batch = batch;
  a.world = (heads + heads_per_rank - 1) / heads_per_rank;
  a.n_local = n_local;
  a.seg_rows = n_local;
  a.heads = heads;
  a.heads_per_rank = heads_per_rank;
  a.head_dim = head_dim;
  a.out_fp32 = out_dtype == PS_B200_FP32;
  return launch_unpack(a, dtype == PS_B200_FP16, static_cast<cudaStream_t>(stream));
}

unsigned long long ps_b200_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------- shared buffers
int ps_b200_shared_alloc(size_t bytes, void** ptr) {
  if (!ptr) return set_error(PS_B200_ERR_INVALID, "null output pointer");
  *ptr = nullptr;
  if (bytes == 0) return set_error(PS_B200_ERR_INVALID, "zero-byte shared buffer");
  if (int rc = check_device()) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_cuda_error("cudaMalloc (shared buffer)", e);
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_cuda_error("cudaMemset (shared buffer)", e);
  }
  *ptr = p;
  return PS_B200_OK;
}

int ps_b200_shared_free(void* ptr) {
  if (!ptr) return PS_B200_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? PS_B200_OK : set_cuda_error("cudaFree (shared buffer)", e);
}

int ps_b200_ipc_export(const void* ptr, unsigned char* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == PS_B200_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return set_error(PS_B200_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return set_cuda_error("cudaIpcGetMemHandle", e);
  std::memcpy(handle, &h, sizeof(h));
  return PS_B200_OK;
}

int ps_b200_ipc_import(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) return set_error(PS_B200_ERR_INVALID, "null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_cuda_error("cudaIpcOpenMemHandle", e);
  *ptr = p;
  return PS_B200_OK;
}

int ps_b200_ipc_close(void* ptr) {
  if (!ptr) return PS_B200_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? PS_B200_OK : set_cuda_error("cudaIpcCloseMemHandle", e);
}

}  // extern "C"

// ------------------------------------------------------------ projection GEMMs
namespace psb {
namespace {

// 2-D map over [rows][cols] 16-bit elements (row stride in elements), box
// 64 columns x box_rows rows, 128-byte swizzle.
int make_map_2d(CUtensorMap* m, const void* base, bool fp16, int64_t cols, int64_t rows, int64_t row_stride,
                unsigned box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(PS_B200_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (row_stride * 2 % 16 != 0 || row_stride <= 0)
    return set_error(PS_B200_ERR_INVALID, "row stride of %lld elements is not a positive multiple of 8",
                     (long long)row_stride);
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(row_stride * 2)};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PS_B200_ERR_INVALID, "cuTensorMapEncodeTiled (2-D) failed with CUresult %d", int(r));
  return PS_B200_OK;
}

// 3-D map over [blocks][rows][cols] (strides in elements), box 64 x 128 x 1.
int make_map_3d(CUtensorMap* m, const void* base, bool fp16, int64_t cols, int64_t rows, int64_t blocks,
                int64_t row_stride, int64_t block_stride) {
  auto fn = encode_fn();
  if (!fn) return set_error(PS_B200_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (row_stride <= 0 || row_stride % 8 != 0 || block_stride <= 0 || block_stride % 8 != 0)
    return set_error(PS_B200_ERR_INVALID, "exchange-buffer strides must be positive multiples of 8 elements");
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(blocks)};
  cuuint64_t strides[2] = {cuuint64_t(row_stride * 2), cuuint64_t(block_stride * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PS_B200_ERR_INVALID, "cuTensorMapEncodeTiled (3-D) failed with CUresult %d", int(r));
  return PS_B200_OK;
}

// 128-row blocks of n GEMM rows, rounded up to whole 256-row pair tiles.
int64_t qkv_rows_blocks(int n) { return 2 * ((int64_t(n) + 255) / 256); }

}  // namespace
}  // namespace psb

extern "C" {

size_t ps_b200_qkv_proj_workspace_bytes(int rows, int heads, int head_dim) {
  if (rows <= 0 || heads <= 0 || head_dim <= 0) return 0;
  const int64_t width = int64_t(heads) * head_dim;
  const int64_t groups = 2 * psb::qkv_rows_blocks(rows);
  const int64_t part = groups * (width / 256) * 128 * 4;
  return static_cast<size_t>(((part + 255) / 256) * 256 + ((groups * 4 + 255) / 256) * 256);
}

int ps_b200_qkv_proj(const void* x, int64_t x_row_stride, const void* w_q, const void* w_k, const void* w_v,
                     const void* b_q, const void* b_k, const void* b_v, int b_dtype, const void* w_qnorm,
                     const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_row_stride,
                     void* const* dst_blocks, int dtype, int world, int n_local, int seg_rows, int heads,
                     int heads_per_rank, int head_dim, int in_features, float eps, void* workspace,
                     size_t workspace_bytes, int* status, void* stream) {
  return ps_b200_qkv_proj_batch(x, x_row_stride, w_q, w_k, w_v, b_q, b_k, b_v, b_dtype, w_qnorm, w_knorm, w_dtype,
                                freqs, 0, freqs_row_stride, dst_blocks, dtype, 1, world, n_local, seg_rows, heads,
                                heads_per_rank, head_dim, in_features, eps, workspace, workspace_bytes, status,
                                stream);
}

int ps_b200_qkv_proj_batch(const void* x, int64_t x_row_stride, const void* w_q, const void* w_k, const void* w_v,
                           const void* b_q, const void* b_k, const void* b_v, int b_dtype, const void* w_qnorm,
                           const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_batch_stride,
                           int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int batch, int world,
                           int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, int in_features,
                           float eps, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  using namespace psb;
  if (!is16bit(dtype)) return set_error(PS_B200_ERR_UNSUPPORTED, "projection supports bf16 and fp16 only");
  if (world < 1 || world > kMaxSegs || n_local < 0 || seg_rows < n_local || heads < 1 || heads_per_rank < 1 ||
      int64_t(heads_per_rank) * world < heads || in_features <= 0 || batch < 0 || freqs_batch_stride < 0 ||
      freqs_batch_stride % 4 != 0)
    return set_error(PS_B200_ERR_INVALID, "inconsistent projection geometry");
  if (int64_t(batch) * n_local >= (int64_t(1) << 31)) return set_error(PS_B200_ERR_UNSUPPORTED, "too many rows");
  if (head_dim != 128) return set_error(PS_B200_ERR_UNSUPPORTED, "projection supports head_dim 128 only");
  const int64_t width = int64_t(heads) * head_dim;
  if (width % 256 != 0) return set_error(PS_B200_ERR_UNSUPPORTED, "projection needs an even head count");
  if (in_features % 64 != 0) return set_error(PS_B200_ERR_UNSUPPORTED, "in_features must be a multiple of 64");
  if (b_dtype != dtype && b_dtype != PS_B200_FP32) return set_error(PS_B200_ERR_UNSUPPORTED, "bias dtype");
  if (w_dtype != dtype && w_dtype != PS_B200_FP32) return set_error(PS_B200_ERR_UNSUPPORTED, "norm weight dtype");
  if (!std::isfinite(eps) || eps < 0.f) return set_error(PS_B200_ERR_INVALID, "eps must be finite and >= 0");
  if (seg_rows == 0 || batch == 0) return PS_B200_OK;
  if (!dst_blocks) return set_error(PS_B200_ERR_INVALID, "null destination table");
  for (int d = 0; d < world; ++d)
    if (!dst_blocks[d] || !aligned16(dst_blocks[d]))
      return set_error(PS_B200_ERR_INVALID, "destination block %d null or not 16-byte aligned", d);
  ProjArgs a{};
  a.n = batch * n_local;
  a.batch = batch;
  a.n_local = n_local;
  a.freqs_batch_stride = batch > 1 ? freqs_batch_stride : 0;
  a.kdim = in_features;
  a.width = static_cast<int>(width);
  a.ntile_n = static_cast<int>(width / 256);
  a.row_blocks = static_cast<int>(qkv_rows_blocks(a.n) / 2);
  a.epi = 1;
  a.bias[0] = b_q;
  a.bias[1] = b_k;
  a.bias[2] = b_v;
  a.bias_fp32 = b_dtype == PS_B200_FP32;
  a.normw[0] = w_qnorm;
  a.normw[1] = w_knorm;
  a.normw_fp32 = w_dtype == PS_B200_FP32;
  a.freqs = freqs;
  a.freqs_row_stride = freqs_row_stride;
  a.eps = eps;
  for (int d = 0; d < world; ++d) a.dst[d] = dst_blocks[d];
  a.world = world;
  a.seg_rows = seg_rows;
  a.heads = heads;
  a.heads_per_rank = heads_per_rank;
  a.head_dim = head_dim;
  a.status = status;
  if (a.n > 0) {
    if (!x || !w_q || !w_k || !w_v || !w_qnorm || !w_knorm || !freqs || !aligned16(x) || !aligned16(w_q) ||
        !aligned16(w_k) || !aligned16(w_v) || !aligned16(w_qnorm) || !aligned16(w_knorm) || !aligned16(freqs) ||
        freqs_row_stride % 4 != 0 || freqs_row_stride < head_dim * 2)
      return set_error(PS_B200_ERR_INVALID, "projection inputs must be non-null and 16-byte aligned");
    for (const void* b : {b_q, b_k, b_v})
      if (b && !aligned16(b)) return set_error(PS_B200_ERR_INVALID, "bias must be 16-byte aligned");
    const size_t need = ps_b200_qkv_proj_workspace_bytes(a.n, heads, head_dim);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return set_error(PS_B200_ERR_INVALID, "projection workspace of %zu bytes required", need);
    if (int rc = check_device()) return rc;
    const bool fp16 = dtype == PS_B200_FP16;
    const int C = proj_clusters(fp16);
    if (C <= 0) return PS_B200_ERR_CUDA;
    const int G = a.ntile_n;
    if (G > C) return set_error(PS_B200_ERR_UNSUPPORTED, "projection width above %d columns", C * 256);
    a.total_groups = 2 * a.row_blocks;
    a.total_tiles = 3 * a.row_blocks * G;  // q, k and v pair tiles, in task order
    a.rounds = static_cast<int>((int64_t(a.total_tiles) + C - 1) / C);
    // Statistics per 128-row block: 2 * total_groups groups (the workspace
    // size above counts the same 2 * qkv_rows_blocks groups).
    const int64_t groups128 = 2 * int64_t(a.total_groups);
    a.ss_part = static_cast<float*>(workspace);
    const int64_t part_bytes = ((groups128 * G * 128 * 4 + 255) / 256) * 256;
    a.counters = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + part_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemsetAsync(a.counters, 0, size_t(groups128) * 4, s);
    if (err != cudaSuccess) return set_cuda_error("projection: clearing the group counters", err);
    CUtensorMap ta, tw[3];
    if (int rc = make_map_2d(&ta, x, fp16, in_features, a.n, x_row_stride, 128)) return rc;
    const void* ws[3] = {w_q, w_k, w_v};
    for (int i = 0; i < 3; ++i)  // each CTA of a pair loads 128 rows of a weight tile
      if (int rc = make_map_2d(&tw[i], ws[i], fp16, in_features, width, in_features, 128)) return rc;
    return launch_proj(ta, tw[0], tw[1], tw[2], a, fp16, C, s);
  }
  // No local rows: only the zero padding of the send blocks.
  if (int rc = check_device()) return rc;
  CUtensorMap none{};
  return launch_proj(none, none, none, none, a, dtype == PS_B200_FP16, 1, static_cast<cudaStream_t>(stream));
}

int ps_b200_out_proj(const void* src, int64_t src_row_stride, int64_t src_block_stride, int src_block_cols,
                     const void* w_o, const void* b_o, int b_dtype, void* out, int64_t out_row_stride, int dtype,
                     int out_dtype, int n_local, int in_features, int out_features, int* status, void* stream) {
  using namespace psb;
  if (!is16bit(dtype)) return set_error(PS_B200_ERR_UNSUPPORTED, "projection supports bf16 and fp16 only");
  if (out_dtype != dtype && out_dtype != PS_B200_FP32)
    return set_error(PS_B200_ERR_UNSUPPORTED, "projection output must be fp32 or the input dtype");
  if (n_local < 0 || in_features <= 0 || out_features <= 0) return set_error(PS_B200_ERR_INVALID, "negative size");
  if (in_features % 64 != 0 || out_features % 256 != 0)
    return set_error(PS_B200_ERR_UNSUPPORTED, "projection needs in_features %% 64 == 0 and out_features %% 256 == 0");
  if (b_dtype != dtype && b_dtype != PS_B200_FP32) return set_error(PS_B200_ERR_UNSUPPORTED, "bias dtype");
  if (n_local == 0) return PS_B200_OK;
  if (!src || !w_o || !out || !aligned16(src) || !aligned16(w_o) || !aligned16(out) || (b_o && !aligned16(b_o)) ||
      out_row_stride % 8 != 0 || out_row_stride < out_features)
    return set_error(PS_B200_ERR_INVALID, "projection buffers must be 16-byte aligned, strides %% 8 == 0");
  const bool blocks = src_block_cols > 0;
  // Blocks may end short of src_block_cols in the last one (padded heads of the
  // NCCL receive layout): the K loop stops at in_features.
  if (blocks && src_block_cols % 64 != 0)
    return set_error(PS_B200_ERR_UNSUPPORTED, "source blocks must hold a multiple of 64 columns");
  if (int rc = check_device()) return rc;
  ProjArgs a{};
  a.n = n_local;
  a.kdim = in_features;
  a.width = out_features;
  a.ntile_n = out_features / 256;
  a.row_blocks = static_cast<int>(qkv_rows_blocks(n_local) / 2);
  a.a_mode = blocks ? 1 : 0;
  a.a_block_k = blocks ? src_block_cols : 0;
  a.epi = 0;
  a.bias[0] = b_o;
  a.bias_fp32 = b_dtype == PS_B200_FP32;
  a.out = out;
  a.out_row_stride = out_row_stride;
  a.out_fp32 = out_dtype == PS_B200_FP32;
  a.status = status;
  a.total_tiles = a.row_blocks * a.ntile_n;
  const bool fp16 = dtype == PS_B200_FP16;
  const int C = proj_clusters(fp16);
  if (C <= 0) return PS_B200_ERR_CUDA;
  a.rounds = (a.total_tiles + C - 1) / C;
  CUtensorMap ta, tw;
  if (blocks) {
    const int64_t nblocks = (in_features + src_block_cols - 1) / src_block_cols;
    if (int rc = make_map_3d(&ta, src, fp16, src_block_cols, n_local, nblocks, src_row_stride, src_block_stride))
      return rc;
  } else {
    if (int rc = make_map_2d(&ta, src, fp16, in_features, n_local, src_row_stride, 128)) return rc;
  }
  if (int rc = make_map_2d(&tw, w_o, fp16, in_features, out_features, in_features, 128)) return rc;
  return launch_proj(ta, tw, tw, tw, a, fp16, C, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
