// Internal declarations shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace psb {

constexpr int kMaxSegs = 64;  // segments (source ranks) per attention call

// Arguments of the attention kernel that are not tensor maps.
struct AttnArgs {
  void* seg_out[kMaxSegs];  // output element (batch 0, row 0, head 0, d 0) of each query segment:
                            // slices of one tensor, or other GPUs' buffers (peer exchange)
  int64_t o_stride[4];   // batch, (unused), row, head strides in elements (d stride 1)
  int seg_rows_q;        // rows allocated per query segment
  int nsegs_q;           // query segments
  int q_tiles_per_seg;   // ceil(seg_rows_q / 128)
  int num_q_tiles;       // prefix tiles + nsegs_q * q_tiles_per_seg
  int seg_rows_k;
  int nsegs_k;
  int num_kv_tiles;      // prefix tiles + sum over key segments of ceil(valid_k / 128)
  int valid_q[kMaxSegs]; // valid rows of each query segment (a prefix of its rows)
  int valid_k[kMaxSegs];
  int group;             // query heads per key/value head (GQA)
  float scale_log2;      // softmax_scale * log2(e)
  int out_fp32;          // 1: output fp32, 0: output in the input 16-bit type
  int* status;           // device status word (0 = ok), may be null
  // Optional prefix range (Flux text tokens): query and key rows [0, pre_len)
  // come from the prefix maps, ahead of the segmented rows; num_q_tiles and
  // num_kv_tiles count both ranges.  pre_len == 0: no prefix.
  int pre_len;
  int pre_tiles;         // ceil(pre_len / 128)
  void* pre_out;         // prefix output row 0, head 0
  int64_t pre_o_stride[4];  // batch, (unused), row, head strides in elements
  // Work units: (query tile pair, head, batch), pair fastest; the grid is 1-D.
  // Units [0, full_units) run whole; each later unit (the last, partial wave)
  // runs as `split` CTAs over consecutive parts of the key range, writing
  // partials that attn_combine_kernel merges.
  int npairs;            // ceil(num_q_tiles / 2)
  int grid_heads;
  int full_units;
  int split;             // 1: no split
  float* ws_o;           // [slot][2][128][128] fp32: O / l of one part, slot = (unit - full_units) * split + part
  float* ws_lse;         // [slot][2][128] fp32: m + log2(l) of one part (log2 units of the scaled scores)
};

constexpr int kMaxSplit = 8;
// Workspace bytes for up to 160 SMs: one partial (O, lse) per CTA of a wave.
constexpr int64_t kAttnWorkspaceBytes = int64_t(160) * 2 * 128 * (128 + 1) * 4;

// Launches the attention grid (full_units + split units * split CTAs) and,
// when units are split, the combine kernel after it on the same stream.
int launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const CUtensorMap& tqp, const CUtensorMap& tkp, const CUtensorMap& tvp,
                     const AttnArgs& args, int64_t total_units, bool fp16, cudaStream_t stream);

// Process-wide count of kernels this library launched (ps_b200_kernel_launches).
void count_launch();

struct PrepassArgs {
  const void* x[3];        // q, k, v projection outputs, [batch][n_local][heads*head_dim]
  int64_t x_batch_stride[3]; // elements between consecutive batch rows
  int64_t x_row_stride[3]; // elements between consecutive tokens
  int64_t x_head_stride[3];// elements between consecutive heads of a token (head_dim: [n][H*D] rows)
  const void* w[2];        // RMSNorm weights of q and k, [heads*head_dim]
  int w_fp32;              // 1: weights are fp32, 0: same 16-bit type as x
  const float* freqs;      // [batch][n_local][head_dim/2][2][2] fp32
  int64_t freqs_batch_stride; // floats between consecutive batch rows (0: one table for the batch)
  int64_t freqs_row_stride;// floats between consecutive tokens
  void* dst[kMaxSegs];     // block [3][batch][seg_rows][heads_per_rank][head_dim] for each destination
                           // rank: slices of the local send buffer, or peers' receive buffers
  int batch, world, n_local, seg_rows, heads, heads_per_rank, head_dim;
  float eps;
  int norm_rope;           // 0: plain pack, 1: full-width RMSNorm + RoPE, 2: per-head RMSNorm + RoPE
  int rope_style;          // 0: interleaved pairs (2j, 2j+1) over the head; 1: split half (j, j+rope_pairs)
  int rope_pairs;          // rotated pairs per head (head_dim/2 for style 0; a multiple of 8 for style 1)
  // Token-mode fan-out (kv_fanout > 0, world 1, heads_per_rank == heads): q rows go to q_out
  // [batch][seg_rows][heads][head_dim]; k and v rows go to each of dst[0..kv_fanout-1], blocks
  // [2][batch][seg_rows][heads][head_dim] (the all-gather of K/V as stores).
  void* q_out;
  int kv_fanout;
};

int launch_prepass(const PrepassArgs& a, bool fp16, cudaStream_t stream);

struct UnpackArgs {
  const void* recv;        // head block src, batch b, row i at recv + src*src_stride + b*batch_stride
                           // + i*row_stride (elements)
  int64_t src_stride, batch_stride, row_stride;
  void* out;               // [batch][n_local][heads][head_dim] (strides below)
  int64_t out_batch_stride;// elements between consecutive batch rows of out
  int64_t out_row_stride;  // elements between consecutive tokens of out
  int batch, world, n_local, seg_rows, heads, heads_per_rank, head_dim;
  int out_fp32;            // 1: write fp32, 0: same 16-bit type as recv
};

int launch_unpack(const UnpackArgs& a, bool fp16, cudaStream_t stream);

// Arguments of the projection GEMMs (proj.cu) that are not tensor maps.
struct ProjArgs {
  int n;                   // rows of A: batch * n_local (epi 1) or this rank's tokens (epi 0)
  int batch;               // epi 1: batch rows; GEMM row m is token m % n_local of batch row m / n_local
  int n_local;             // epi 1: tokens per batch row
  int64_t freqs_batch_stride;  // epi 1: floats between the rotation tables of batch rows (0: shared)
  int kdim;                // K: input features (a multiple of 64)
  int width;               // output features of one projection (a multiple of 256)
  int ntile_n;             // width / 256: column tiles of one projection
  int row_blocks;          // ceil(n / 256): row blocks of the 256-row pair tiles
  int a_mode;              // 0: A is [n][kdim] rows; 1: A is [src][n][a_block_k] blocks (k = src*a_block_k + c)
  int a_block_k;           // columns per source block (a multiple of 64) for a_mode 1
  int epi;                 // 0: y = A W^T + b stored row-major; 1: q/k/v with RMSNorm, RoPE and the Ulysses pack
  const void* bias[3];     // per projection, [width], may be null
  int bias_fp32;           // 1: fp32 biases, 0: the 16-bit activation type
  const void* normw[2];    // RMSNorm weights of q and k, [width]
  int normw_fp32;
  const float* freqs;      // [n][head_dim/2][2][2] rotation table
  int64_t freqs_row_stride;
  float eps;
  void* dst[kMaxSegs];     // epi 1: destination d's block [3][batch][seg_rows][heads_per_rank][head_dim]
  int world, seg_rows, heads, heads_per_rank, head_dim;
  void* out;               // epi 0: [n][width] (row stride out_row_stride elements)
  int64_t out_row_stride;
  int out_fp32;
  // Scheduling (persistent CTA pairs, one task = one 256 x 256 pair tile per round):
  int total_groups;        // epi 1: 2 * row_blocks q/k groups of pair tiles
  int total_tiles;         // epi 0: row_blocks * ntile_n; epi 1: 3 * row_blocks * ntile_n
  int rounds;
  // RMSNorm statistics per 128-row block (two per pair row block):
  float* ss_part;          // epi 1: [4 * row_blocks][ntile_n][128] partial sums of squares
  unsigned* counters;      // epi 1: [4 * row_blocks] tiles that posted their partials (zeroed)
  int* status;             // device status word, may be null
};

// Launches the projection GEMM: `clusters` pairs of CTAs (cooperative
// cluster launch: every CTA resident, one per SM).
int launch_proj(const CUtensorMap& ta, const CUtensorMap& tw0, const CUtensorMap& tw1, const CUtensorMap& tw2,
                const ProjArgs& args, bool fp16, int clusters, cudaStream_t stream);
// CTA pairs the device keeps resident at once (0 on error, recorded).
int proj_clusters(bool fp16);

struct BroadcastArgs {
  const void* src;         // 16-byte vectors to copy
  void* dst[kMaxSegs];     // destinations (this GPU's memory or a peer's)
  int ndst;
  int64_t vectors;
};

int launch_broadcast(const BroadcastArgs& a, cudaStream_t stream);

// Error bookkeeping (thread-local message, returned code).
int set_error(int code, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t err);

}  // namespace psb
