/*
 * ps_b200.h - C ABI of the B200 (sm_100a) Ulysses sequence-parallel attention
 * provider for ComfyUI-PowerShard.
 *
 * The library (libps_b200.so) holds hand-written CUDA kernels for the three
 * device steps of PowerShard's Ulysses self-attention block.  The two
 * all-to-all exchanges between them are either issued by the host (NCCL
 * through torch.distributed, between ps_b200_prepass / ps_b200_ulysses_attn_fwd
 * / ps_b200_unpack), or fused into the kernels over NVLink peer memory: the
 * pre-pass stores each destination's block straight into that rank's receive
 * buffer (ps_b200_prepass_to) and the attention epilogue stores each output
 * row straight into its owner's staging buffer (ps_b200_ulysses_attn_to);
 * the host then only orders the steps across ranks (two 4-byte all-reduces).
 * Every compute entry point takes plain device pointers, sizes and a
 * cudaStream_t (as void*), launches asynchronously on that stream and returns
 * a status code; only ps_b200_shared_alloc allocates device memory.
 *
 * Reference interfaces replaced (paths inside the ComfyUI-PowerShard tree):
 *   ps_b200_prepass        powershard/wan_model.py:421-430 (attention_qkv:
 *                          norm_q/norm_k RMSNorm + rope_apply) fused with the
 *                          send-side packing of ulysses_to_sequence,
 *                          wan_model.py:343-361 / attention.py:57-75.
 *   ps_b200_attn_fwd       the provider call of AttentionDispatcher.__call__,
 *                          powershard/attention_policy.py:101-149 (semantics of
 *                          attention_contract.py:85-145, non-causal, no mask).
 *   ps_b200_ulysses_attn_fwd  the same attention reading the receive buffer of
 *                          ulysses_to_sequence in place (wan_model.py:362-364)
 *                          and writing the send buffer of ulysses_to_heads
 *                          (wan_model.py:373-376).
 *   ps_b200_unpack         receive-side unpack of ulysses_to_heads,
 *                          powershard/wan_model.py:377-380 / attention.py:93-95.
 *   ps_b200_prepass_to, ps_b200_ulysses_attn_to, ps_b200_unpack_strided,
 *   ps_b200_shared_alloc/free, ps_b200_ipc_export/import/close
 *                          the same steps with the two all_to_all_single calls
 *                          of wan_model.py:360 and :376 replaced by peer
 *                          stores (no reference counterpart for the buffer
 *                          sharing itself: NCCL owns it there).
 *   ps_b200_ulysses_joint_attn_fwd, ps_b200_ulysses_joint_attn_to,
 *   ps_b200_broadcast       the attention of image_parallel.SequenceAttention
 *                          (powershard/image_parallel.py:96-110: replicated
 *                          text rows + split image rows), computed on the
 *                          Ulysses exchange instead of the reference's K/V
 *                          all-gather; the broadcast all-gathers text outputs.
 *   ps_b200_prepass rope_style 1   rope_split_half of the H3 path,
 *                          powershard/attention.py:98-103.
 *   ps_b200_qkv_proj       the q/k/v Linear layers of attention_qkv
 *                          (wan_model.py:425-429, self.q/k/v) as one GEMM whose
 *                          epilogue also does norm_q/norm_k, rope_apply and the
 *                          send-side pack (the whole of ps_b200_prepass).
 *   ps_b200_out_proj       self.o (wan_model.py:438) reading the attention
 *                          output from the exchange buffer in place: the
 *                          receive-side unpack of ulysses_to_heads
 *                          (wan_model.py:377-380) fused into the GEMM.
 *   ps_b200_prepass_batch, ps_b200_ulysses_attn_batch, ps_b200_unpack_batch
 *                          the same three steps for a batch of rows (CFG) in
 *                          one exchange, as the reference packs it: send
 *                          [W, T, B, width, h, D] (wan_model.py:350-362) and
 *                          output send [W, B, width, h, D] (:373-378).
 *   ps_b200_kernel_launches, ps_b200_selftest_bounded_wait,
 *   ps_b200_block_fwd_static  no reference counterpart (instrumentation,
 *                          failure-detection self-test, allocation-free block).
 *
 * Layout vocabulary: a "segmented" tensor is [batch][segment][row][head][d]
 * with arbitrary element strides for the first four axes and d contiguous.
 * Rows of segment s are valid while s*seg_rows + row < len; the Ulysses
 * receive buffer is one segment per source rank.
 */
#ifndef PS_B200_H
#define PS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PS_B200_ABI_VERSION 4

/* Return codes. */
#define PS_B200_OK 0
#define PS_B200_ERR_INVALID 1     /* bad pointer / size / stride / alignment      */
#define PS_B200_ERR_UNSUPPORTED 2 /* valid request outside what the kernels cover */
#define PS_B200_ERR_CUDA 3        /* CUDA runtime or driver error                  */

/* Element types. */
#define PS_B200_BF16 0
#define PS_B200_FP16 1
#define PS_B200_FP32 2

/* Device status codes written to *status by the attention kernel when one of
 * its bounded internal waits expires (the launch then returns early, the
 * output is undefined and the host must raise).  0 means success. */
#define PS_B200_DEVICE_TIMEOUT_FIRST 101
#define PS_B200_DEVICE_TIMEOUT_LAST 199

/*
 * Attention workspace.  Every attention entry point takes an optional device
 * workspace (16-byte aligned, >= PS_B200_ATTN_WORKSPACE_BYTES; NULL or smaller
 * disables its use).  With one, the units of work of the last, partial wave
 * (a unit is two 128-row query tiles of one head) are split along the key
 * range over several CTAs whose partial results (O / l in fp32 and the
 * log-sum-exp of each row) a second kernel merges, so that wave finishes
 * sooner; results equal the unsplit computation up to fp32 rounding.  The
 * workspace is scratch owned by one call at a time: calls that may overlap
 * on the GPU need separate workspaces.  Size: one partial per CTA of a wave
 * for up to 160 SMs.
 */
#define PS_B200_ATTN_WORKSPACE_BYTES (160LL * 2 * 128 * 129 * 4)

/* Kernels this library has launched in this process (all entry points). */
unsigned long long ps_b200_kernel_launches(void);

/* ABI version of the loaded library (PS_B200_ABI_VERSION). */
int ps_b200_abi_version(void);

/* Message of the last error returned on the calling host thread. */
const char* ps_b200_last_error(void);

/*
 * Fused q/k RMSNorm + RoPE + Ulysses pack (replaces attention_qkv plus the
 * send-side packing of ulysses_to_sequence).
 *   x_q, x_k, x_v  [n_local][heads][head_dim] projection outputs (dtype), row
 *                  strides x_row_strides[0..2] and head strides
 *                  x_head_strides[0..2] in elements (multiples of 8; NULL
 *                  head strides = head_dim, i.e. [n_local][heads*head_dim]
 *                  rows; head stride L*head_dim reads a [heads][L][head_dim]
 *                  tensor, ComfyUI's skip_reshape layout).
 *   w_qnorm, w_knorm RMSNorm weights, w_dtype = dtype or FP32: [heads*head_dim]
 *                  for norm_rope 1, [head_dim] (shared by all heads) for 2.
 *   freqs          [n_local][head_dim/2][2][2] fp32 rotation table (the
 *                  reference's freqs[0, :, 0]), freqs_row_stride in floats.
 *   send           [world][3][seg_rows][heads_per_rank][head_dim] (dtype).
 *   norm_rope      1: RMSNorm over the full width + RoPE on q and k (Wan),
 *                  2: RMSNorm over each head + RoPE (Flux / H3 QK-norm), 0: pack only.
 *   rope_style     0: interleaved pairs (2j, 2j+1), rope_pairs = head_dim/2
 *                  (powershard/wan_model.py:325-329); 1: split half, pairs
 *                  (j, j+rope_pairs) for j < rope_pairs, elements >= 2*rope_pairs
 *                  unrotated (H3 partial RoPE, powershard/attention.py:98-103;
 *                  rope_pairs a multiple of 8).  freqs rows hold rope_pairs
 *                  2x2 matrices.
 * Rows n_local..seg_rows-1 and heads heads..world*heads_per_rank-1 of the
 * send buffer are written as zeros.
 */
int ps_b200_prepass(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                    const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                    const float* freqs, int64_t freqs_row_stride, void* send, int dtype, int world, int n_local,
                    int seg_rows, int heads, int heads_per_rank, int head_dim, float eps, int norm_rope,
                    int rope_style, int rope_pairs, void* stream);

/*
 * softmax(Q K^T * softmax_scale) V over segmented tensors (BLHD is the case
 * segs = 1, seg_rows = len).  q/k/v/out strides are {batch, segment, row,
 * head} in elements; all must be multiples of 8 elements and pointers 16-byte
 * aligned.  dtype BF16 or FP16 for q/k/v, out_dtype = dtype or FP32; head_dim 128;
 * heads_q % heads_kv == 0 (GQA).  status: device int (may be NULL) that
 * receives a PS_B200_DEVICE_TIMEOUT_* code if the kernel aborts.
 */
int ps_b200_attn_fwd(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                     const void* v, const int64_t v_strides[4], void* out, const int64_t out_strides[4],
                     int dtype, int out_dtype, int batch, int heads_q, int heads_kv, int head_dim, int seg_rows_q,
                     int segs_q, int len_q, int seg_rows_k, int segs_k, int len_k, float softmax_scale,
                     void* workspace, size_t workspace_bytes, int* status, void* stream);

/*
 * Attention over the Ulysses receive buffer recv [world][3][seg_rows][heads_per_rank][head_dim]
 * for heads 0..heads_valid-1 of this rank, sequence length `total`; the
 * result goes to out_send [world][seg_rows][heads_per_rank][head_dim], the
 * send buffer of the inverse all-to-all (rows >= the destination's valid
 * rows and heads >= heads_valid are left untouched).  out_dtype = dtype or
 * FP32 (then out_send holds fp32 elements).  seg_valid: host array of
 * `world` ints, the valid rows of each source segment (at most seg_rows each,
 * summing to total; at most 64 segments), or NULL for ceil-width token shards
 * (segment s holds min(seg_rows, max(0, total - s*seg_rows)) rows, the
 * split of shard_bounds, powershard/config.py:107-112).  An explicit table
 * serves the balanced split of the image Layout
 * (powershard/image_layout.py:12-15), whose padding rows may sit in middle
 * segments.
 */
int ps_b200_ulysses_attn_fwd(const void* recv, void* out_send, int dtype, int out_dtype, int world, int seg_rows,
                             int total, const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                             float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                             void* stream);

/*
 * Joint attention (Flux: text tokens replicated on every rank, image tokens
 * Ulysses-split): keys and queries are the rank's text rows prefix_qkv
 * [3][prefix_len][heads_per_rank][head_dim] followed by the image rows of the
 * receive buffer recv (as in ps_b200_ulysses_attn_fwd).  Text query outputs
 * go to prefix_out [prefix_len][heads_per_rank][head_dim], image query
 * outputs to out_send.  seg_valid as in ps_b200_ulysses_attn_fwd (the
 * image Layout's balanced split, or NULL for ceil-width shards).  No
 * counterpart call in the reference, which
 * all-gathers K/V for this model (powershard/image_parallel.py:96-110); the
 * result equals attention over [text; image] (ComfyUI Flux joint attention).
 */
int ps_b200_ulysses_joint_attn_fwd(const void* recv, const void* prefix_qkv, void* out_send, void* prefix_out,
                                   int dtype, int out_dtype, int world, int seg_rows, int total, int prefix_len,
                                   const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                                   float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                                   void* stream);

/*
 * Inverse unpack: recv [world][seg_rows][heads_per_rank][head_dim] (dtype)
 * -> out [n_local][heads][head_dim] (out_dtype = dtype or FP32), token row
 * stride out_row_stride elements.  Padded heads are dropped.
 */
int ps_b200_unpack(const void* recv, void* out, int64_t out_row_stride, int dtype, int out_dtype, int world,
                   int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, void* stream);

/*
 * Unpack with explicit input strides: head block src, token row i of recv
 * starts at recv + src*src_stride + i*row_stride elements (head j of the
 * block at + j*head_dim).  ps_b200_unpack is the case src_stride =
 * seg_rows*heads_per_rank*head_dim, row_stride = heads_per_rank*head_dim;
 * the peer-exchange staging buffer [seg_rows][world*heads_per_rank][head_dim]
 * is src_stride = heads_per_rank*head_dim, row_stride =
 * world*heads_per_rank*head_dim.
 */
int ps_b200_unpack_strided(const void* recv, int64_t src_stride, int64_t row_stride, void* out,
                           int64_t out_row_stride, int dtype, int out_dtype, int n_local, int heads,
                           int heads_per_rank, int head_dim, void* stream);

/* ------------------------------------------------------------------------
 * Peer-memory exchange (one process per GPU, GPUs of one node with NVLink
 * peer access).  Each rank allocates its receive buffer
 * [world][3][seg_rows][heads_per_rank][head_dim] and its output staging
 * buffer [seg_rows][world*heads_per_rank][head_dim] with ps_b200_shared_alloc,
 * exports them with ps_b200_ipc_export, gathers the peers' handles (any host
 * transport) and maps them with ps_b200_ipc_import.  Per step:
 *   ps_b200_prepass_to(dst_blocks[d] = receive buffer of rank d + rank*block)
 *   -> all ranks' pre-passes finished (a cross-rank barrier on the stream)
 *   -> ps_b200_ulysses_attn_to(out_blocks[s] = staging buffer of rank s +
 *      rank*heads_per_rank*head_dim, out_row_stride = world*heads_per_rank*head_dim)
 *   -> barrier -> ps_b200_unpack_strided(own staging buffer).
 * The barriers also keep a rank from overwriting a peer buffer that the peer
 * still reads.  Visibility comes from stream order: a barrier (e.g. a
 * 4-byte all-reduce) starts after the storing kernel has completed, and a
 * completed kernel's stores, peer stores included, are visible system-wide.
 * ---------------------------------------------------------------------- */
#define PS_B200_IPC_HANDLE_BYTES 64

/* cudaMalloc + zero fill of `bytes` (the allocation base, as IPC requires). */
int ps_b200_shared_alloc(size_t bytes, void** ptr);
int ps_b200_shared_free(void* ptr);
/* Handle (PS_B200_IPC_HANDLE_BYTES bytes) of a ps_b200_shared_alloc buffer. */
int ps_b200_ipc_export(const void* ptr, unsigned char* handle);
/* Map a peer's buffer into this process (peer access enabled lazily). */
int ps_b200_ipc_import(const unsigned char* handle, void** ptr);
int ps_b200_ipc_close(void* ptr);

/*
 * ps_b200_prepass with one destination pointer per rank instead of one send
 * buffer: dst_blocks[d] (16-byte aligned, possibly another GPU's memory)
 * receives the [3][seg_rows][heads_per_rank][head_dim] block of destination d.
 */
int ps_b200_prepass_to(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                       const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                       const float* freqs, int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int world,
                       int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, float eps,
                       int norm_rope, int rope_style, int rope_pairs, void* stream);

/*
 * Token mode with the K/V all-gather as stores: the pre-pass of this rank's
 * n_local rows (as ps_b200_prepass, world 1, all heads) writes q to q_out
 * [width][heads][head_dim] and k, v to each of the ndst (1..64) blocks
 * kv_dst[d], [2][width][heads][head_dim] (rank d's gathered K/V, slot of
 * this rank; possibly another GPU's memory).  Rows n_local..width-1 are
 * zeros.  Replaces the pack + gather_tokens of wan_model.py:489-500.
 */
int ps_b200_prepass_token_to(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                             const int64_t x_head_strides[3], const void* w_qnorm, const void* w_knorm, int w_dtype,
                             const float* freqs, int64_t freqs_row_stride, void* q_out, void* const* kv_dst,
                             int ndst, int dtype, int n_local, int width, int heads, int head_dim, float eps,
                             int norm_rope, int rope_style, int rope_pairs, void* stream);

/*
 * Joint attention (as ps_b200_ulysses_joint_attn_fwd) with the image outputs
 * stored through one pointer per source segment (row stride out_row_stride
 * elements, head j at + j*head_dim): the peer exchange's staging buffers.
 * Text outputs go to prefix_out as there.
 */
int ps_b200_ulysses_joint_attn_to(const void* recv, const void* prefix_qkv, void* const* out_blocks,
                                  int64_t out_row_stride, void* prefix_out, int dtype, int out_dtype, int world,
                                  int seg_rows, int total, int prefix_len, const int* seg_valid, int heads_per_rank,
                                  int heads_valid, int head_dim, float softmax_scale, void* workspace,
                                  size_t workspace_bytes, int* status, void* stream);

/*
 * Copies `bytes` (a multiple of 16, 16-byte aligned) from src to each of the
 * ndst (1..64) destinations, which may be other GPUs' memory: the all-gather
 * of the text outputs in the peer exchange of joint attention.
 */
int ps_b200_broadcast(void* const* dst, int ndst, const void* src, size_t bytes, void* stream);

/*
 * ps_b200_ulysses_attn_fwd with one output pointer per source segment: valid
 * row i of segment s, head j goes to out_blocks[s] + i*out_row_stride +
 * j*head_dim elements (out_dtype), possibly another GPU's memory.
 */
int ps_b200_ulysses_attn_to(const void* recv, void* const* out_blocks, int64_t out_row_stride, int dtype,
                            int out_dtype, int world, int seg_rows, int total, const int* seg_valid,
                            int heads_per_rank, int heads_valid, int head_dim, float softmax_scale, void* workspace,
                            size_t workspace_bytes, int* status, void* stream);

/*
 * Batched Ulysses steps: B rows of a batch (e.g. the CFG pair) go through one
 * exchange, in the reference's packing (powershard/wan_model.py:350-362 and
 * :373-378).  The existing entry points are the case batch = 1.
 *
 * ps_b200_prepass_batch: as ps_b200_prepass_to for rows b = 0..batch-1.  Row
 *   (b, i) of x_* starts at x_* + b*x_batch_strides[.] + i*x_row_strides[.]
 *   elements; its rotation table at freqs + b*freqs_batch_stride +
 *   i*freqs_row_stride floats (freqs_batch_stride 0: one table for every
 *   row).  dst_blocks[d] receives destination d's block
 *   [3][batch][seg_rows][heads_per_rank][head_dim] (a slice of the local send
 *   buffer [world][3][batch][seg_rows][h][D], or a peer's receive buffer).
 */
int ps_b200_prepass_batch(const void* x_q, const void* x_k, const void* x_v, const int64_t x_batch_strides[3],
                          const int64_t x_row_strides[3], const int64_t x_head_strides[3], const void* w_qnorm,
                          const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_batch_stride,
                          int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int batch, int world,
                          int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, float eps,
                          int norm_rope, int rope_style, int rope_pairs, void* stream);

/*
 * ps_b200_ulysses_attn_batch: attention over the batched receive buffer recv
 *   [world][3][batch][seg_rows][heads_per_rank][head_dim]; valid row i of
 *   segment s, batch row b, head j goes to out_blocks[s] + b*out_batch_stride
 *   + i*out_row_stride + j*head_dim elements (out_dtype): the batched output
 *   send buffer [world][batch][seg_rows][h][D] (out_blocks[s] = its slice s,
 *   batch stride seg_rows*h*D, row stride h*D), the owners' staging buffers
 *   [batch][seg_rows][world*h][D] of the peer exchange, or at world 1 the
 *   final [batch][n][heads][head_dim] output.
 */
int ps_b200_ulysses_attn_batch(const void* recv, void* const* out_blocks, int64_t out_batch_stride,
                               int64_t out_row_stride, int dtype, int out_dtype, int batch, int world, int seg_rows,
                               int total, const int* seg_valid, int heads_per_rank, int heads_valid, int head_dim,
                               float softmax_scale, void* workspace, size_t workspace_bytes, int* status,
                               void* stream);

/*
 * ps_b200_unpack_batch: as ps_b200_unpack_strided for batch rows; row i of
 *   batch row b, head block src at recv + src*src_stride + b*batch_stride +
 *   i*row_stride elements, written to out + b*out_batch_stride +
 *   i*out_row_stride (+ head*head_dim).
 */
int ps_b200_unpack_batch(const void* recv, int64_t src_stride, int64_t batch_stride, int64_t row_stride, void* out,
                         int64_t out_batch_stride, int64_t out_row_stride, int dtype, int out_dtype, int batch,
                         int n_local, int heads, int heads_per_rank, int head_dim, void* stream);

/*
 * Projection GEMMs (tcgen05.mma.cta_group::2 on 256x256 tiles, one persistent
 * pair of CTAs per two SMs, cooperative cluster launch: the grid is every pair
 * the device keeps resident, so nothing else should hold SMs the call needs).
 *
 * ps_b200_qkv_proj: q|k|v = x [W_q|W_k|W_v]^T + b for this rank's n_local
 *   tokens, x [n_local][in_features] (row stride x_row_stride), weights
 *   [heads*head_dim][in_features] row-major (PyTorch Linear), biases b_*
 *   [heads*head_dim] (b_dtype = dtype or FP32; NULL = none).  The q and k
 *   outputs are RMS-normalised over the full width (eps, weights w_qnorm /
 *   w_knorm), rotated by freqs [n_local][head_dim/2][2][2] and, with v, stored
 *   as ps_b200_prepass_to stores them: dst_blocks[d] receives destination
 *   d's [3][seg_rows][heads_per_rank][head_dim] block, padding rows and head
 *   slots zeroed.  The projections themselves never reach memory.  The RMS
 *   statistic is taken over the fp32 accumulator (not a rounded projection).
 *   head_dim 128, heads even, in_features % 64 == 0.  workspace: device
 *   scratch of ps_b200_qkv_proj_workspace_bytes(batch * n_local, heads, head_dim)
 *   bytes (per-row partial sums of squares and group counters), owned by one
 *   call at a time.  status: device int (may be NULL) receiving a
 *   PS_B200_DEVICE_TIMEOUT_* code if a bounded wait expires.
 */
size_t ps_b200_qkv_proj_workspace_bytes(int rows, int heads, int head_dim);
int ps_b200_qkv_proj(const void* x, int64_t x_row_stride, const void* w_q, const void* w_k, const void* w_v,
                     const void* b_q, const void* b_k, const void* b_v, int b_dtype, const void* w_qnorm,
                     const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_row_stride,
                     void* const* dst_blocks, int dtype, int world, int n_local, int seg_rows, int heads,
                     int heads_per_rank, int head_dim, int in_features, float eps, void* workspace,
                     size_t workspace_bytes, int* status, void* stream);

/*
 * ps_b200_qkv_proj_batch: ps_b200_qkv_proj for a batch of rows (CFG) in one
 *   GEMM: x holds batch * n_local rows (batch row b's tokens at rows
 *   b*n_local ...), the rotation table of batch row b at freqs +
 *   b*freqs_batch_stride floats (0: one table), and destination d's block is
 *   [3][batch][seg_rows][heads_per_rank][head_dim] (the batched send layout of
 *   ps_b200_prepass_batch).  ps_b200_qkv_proj is the case batch = 1.
 */
int ps_b200_qkv_proj_batch(const void* x, int64_t x_row_stride, const void* w_q, const void* w_k, const void* w_v,
                           const void* b_q, const void* b_k, const void* b_v, int b_dtype, const void* w_qnorm,
                           const void* w_knorm, int w_dtype, const float* freqs, int64_t freqs_batch_stride,
                           int64_t freqs_row_stride, void* const* dst_blocks, int dtype, int batch, int world,
                           int n_local, int seg_rows, int heads, int heads_per_rank, int head_dim, int in_features,
                           float eps, void* workspace, size_t workspace_bytes, int* status, void* stream);

/*
 * ps_b200_out_proj: out = A W_o^T + b_o, out [n_local][out_features]
 *   (out_dtype = dtype or FP32, row stride out_row_stride), W_o
 *   [out_features][in_features].  A row i is read in place from the
 *   exchange buffer that holds the attention output:
 *     src_block_cols == 0: src row i at src + i*src_row_stride (the peer
 *       exchange's staging buffer [seg_rows][world*h][head_dim]: row stride
 *       world*h*head_dim, its first heads*head_dim columns are the heads in
 *       order);
 *     src_block_cols > 0: columns [b*src_block_cols, (b+1)*src_block_cols) of
 *       row i at src + b*src_block_stride + i*src_row_stride (the NCCL
 *       receive buffer [world][seg_rows][h][head_dim]: block stride
 *       seg_rows*h*head_dim, row stride and block width h*head_dim).
 *   in_features % 64 == 0, out_features % 256 == 0, 16-byte aligned buffers.
 */
int ps_b200_out_proj(const void* src, int64_t src_row_stride, int64_t src_block_stride, int src_block_cols,
                     const void* w_o, const void* b_o, int b_dtype, void* out, int64_t out_row_stride, int dtype,
                     int out_dtype, int n_local, int in_features, int out_features, int* status, void* stream);

/*
 * Self-test of the bounded waits (no counterpart in the reference): one warp
 * waits on an mbarrier nothing arrives on for limit_us microseconds (1 ..
 * 2e6), then writes PS_B200_DEVICE_TIMEOUT_LAST to *status (device int) and
 * exits; the context stays usable.  Used by the failure-detection tests.
 */
int ps_b200_selftest_bounded_wait(int* status, int limit_us, void* stream);

/*
 * Single-GPU self-attention block that allocates nothing (no counterpart in
 * the reference).  For callers that may not allocate device memory while
 * they run - e.g. a plugin host that owns the device-memory budget through
 * its own pool, or a step that must not hit cudaMalloc's implicit device
 * synchronisation.  Same math as ps_b200_prepass (world 1, norm_rope 1)
 * followed by ps_b200_ulysses_attn_fwd (world 1): out [n][heads][head_dim]
 * in out_dtype, head_dim 128 only.  Its scratch (packed q/k/v and the status
 * word) is a fixed 96 MiB static device array, so 6 * n * heads * head_dim
 * <= 96 MiB (n * heads <= 131072 at head_dim 128); larger requests return
 * PS_B200_ERR_UNSUPPORTED before any work is queued.  A GPU holds the array
 * from the first call on it (with CUDA_MODULE_LOADING=EAGER: from the
 * creation of the process's context on it) until the process exits.  The
 * first call on a device (and the first after that device's context was
 * reset) looks up the array's device address (cudaGetSymbolAddress), so
 * make it before any stream capture.  Calls share the array: calls that
 * overlap on the GPU race.  If host_status is not NULL the call synchronizes
 * the stream and stores the kernel's device status there (0 = ok).  With
 * NULL it stays asynchronous and reports no device-side abort: the status
 * word lives in the shared array and the next call clears it.
 */
int ps_b200_block_fwd_static(const void* x_q, const void* x_k, const void* x_v, const int64_t x_row_strides[3],
                             const void* w_qnorm, const void* w_knorm, int w_dtype, const float* freqs,
                             int64_t freqs_row_stride, void* out, int dtype, int out_dtype, int n, int heads,
                             int head_dim, float eps, float softmax_scale, int* host_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PS_B200_H */
