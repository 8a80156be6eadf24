// Host-side declarations of the sm_100a kernels' launchers.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace laya {

// ---- tcgen05 GEMM: out = epilogue(A[M,K] . W[N,K]^T) ------------------------
// A 2-CTA cluster computes a kGemmBM x kGemmBN tile; each CTA loads 128 rows of
// A (TMA box 64 x 128) and kGemmBN/2 rows of W (box 64 x kGemmBN/2).
constexpr int kGemmBM = 256;
constexpr int kGemmBN = 256;
constexpr int kGemmBK = 64;
constexpr int kGemmABoxRows = 128;
constexpr int kGemmBBoxRows = kGemmBN / 2;
// Narrow 256 x 128 tiles for N = 1024 outputs: twice the tiles per wave.
constexpr int kGemmBNNarrow = 128;
constexpr int kGemmBBoxRowsNarrow = kGemmBNNarrow / 2;
// Output tiles leave through 32-row TMA boxes of 128 bytes per row:
// 64 f16 columns or 32 f32 columns.
constexpr int kGemmOutBoxRows = 32;
// The scorer epilogue leaves one partial dot product per (256-column tile,
// column half) of its 1024 outputs.
constexpr int kScorerPartials = 2 * (1024 / kGemmBN);

enum GemmEpilogue : int {
  kEpiQkvRope = 0,  // f16 out [M, 3072]; RoPE (rotate-half) on q,k; q,k scaled
  kEpiQkvBias = 1,  // f16 out [M, 3072]; + bias; q,k scaled (head layers, no RoPE)
  kEpiResid = 2,    // f32 x[M, N] += acc (+ bias)
  kEpiGeglu = 3,    // f16 out [M, n_valid]; tile = 128 gate | 128 up columns
  kEpiBiasRelu = 4, // f16 out [M, N] = relu(acc + bias)
  kEpiScorer = 5,   // f32 partial[N/256][ldo] = sum_c gelu(acc + bias) * wvec
  kEpiStoreF32 = 6, // f32 out [M, N] = acc (tests)
  // split-K partial sums: the K range is cut into `splits` parts and part s of
  // tile (m, n) stores its f32 sum at output rows s * split_rows + m (part 0
  // adds `bias`, if any).  A row kernel adds the parts to the residual in part
  // order (deterministic), so small-M GEMMs spread their K loop over more SMs.
  kEpiPartial = 7,
  // residual GEMM whose tiles do not fill the last wave: work units below
  // main_tiles are whole tiles reduce-added into x (as kEpiResid, + bias);
  // the remaining tiles (whole row blocks from tail_row0 on) are cut into
  // `splits` K parts each, and part s of a tile stores its f32 sum at rows
  // s * split_rows + (row - tail_row0) of the second output map (the parts
  // region), for the next LayerNorm to add in part order
  kEpiResidTail = 8,
};

struct GemmArgs {
  int M;               // valid rows of A and of the output
  int N;               // rows of W (multiple of 256)
  int K;               // multiple of 64
  int* err;            // device error word
  void* out;
  int ldo;             // output leading dimension in elements
  const float* bias;   // [N] or nullptr
  const int* pos;      // per-row RoPE position
  const float* cosb;   // [max_len][32]
  const float* sinb;   // [max_len][32]
  float scale;         // q/k scale
  const float* wvec;   // scorer output weights [N]
  int n_valid;         // valid output columns for kEpiGeglu
  int splits;          // kEpiPartial / kEpiResidTail: K parts (>= 1)
  int split_rows;      // kEpiPartial: output rows per part (multiple of 256, >= M);
                       // kEpiResidTail: the same for the tail rows (>= M - tail_row0)
  int main_tiles;      // kEpiResidTail: tiles reduce-added whole (a multiple of N / 256)
  int tail_row0;       // kEpiResidTail: first row of the split tiles (main_tiles / (N / 256) * 256)
  unsigned long long wait_limit_ns;  // 0: the default bound (2 s)
  int stuck;           // timeout test: the producers first wait on a barrier nothing completes
};

// Encodes a 2-D f16 K-major tensor map: rows x k elements, row stride k*2 B,
// box {64, box_rows}, 128-byte swizzle.  Returns 0 on success.
int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k,
                  uint32_t box_rows);
// General 2-D row-major map (f16 or f32) with a 128-byte-wide box
// (box_cols * element size == 128) and 128-byte swizzle.
int make_tmap_2d(CUtensorMap* map, const void* base, bool f32, uint64_t rows, uint64_t cols,
                 uint32_t box_cols, uint32_t box_rows);

// Tensor maps of one GEMM: A operand (box 64 x kGemmABoxRows), weights
// (box 64 x kGemmBBoxRows) and the output (box 128 B x kGemmOutBoxRows; any
// valid map for kEpiScorer, which writes through `out` directly).
struct GemmMaps {
  const CUtensorMap* a;
  const CUtensorMap* b;
  const CUtensorMap* out;
  const CUtensorMap* out2 = nullptr;  // kEpiResidTail: the parts region
};

// bn: kGemmBN, or kGemmBNNarrow for kEpiResid / kEpiStoreF32 (then the
// weight map's box has kGemmBNNarrow / 2 rows).
cudaError_t launch_gemm(int epilogue, const GemmMaps& maps, const GemmArgs& args, int num_sms,
                        cudaStream_t stream, int bn = kGemmBN);

// ---- attention over compacted sequences ----------------------------------------
// Sequences longer than kAttnTcQRows (128) tokens: work items of at most 128
// query rows of one sequence, int4 (first query row, query rows, first row
// of the sequence, sequence length), one per 128-row block.  Items whose
// queries see more key blocks come first.  q/k/v rows are loaded in boxes of
// kAttnTcBoxRows rows, only those of the item's sequence.
constexpr int kAttnTcQRows = 128;
constexpr int kAttnTcBoxRows = 32;
struct AttnArgs {
  __half* out;            // [R, 1024] context, token-major
  const int4* items;      // [num_items]
  int num_items;
  int window;             // < 0: global
  int* err;               // device error word
  unsigned long long wait_limit_ns;  // 0: the default bound (2 s)
  int stuck;              // timeout test: the producer first waits on a barrier nothing completes
};
// Sequences of at most kAttnTcQRows tokens: tiles (first row, rows) packing
// whole consecutive sequences; units (tile, head), single pass, four in
// flight per SM on a persistent grid of min(16 * num_tiles, num_sms) CTAs;
// each row sees only its own sequence (rowseq, seq_start, seq_len).  tm_qkv
// is the same map as the flash kernel's (box 64 columns x kAttnTcBoxRows
// rows).
struct AttnShortArgs {
  __half* out;            // [R, 1024]
  const int2* tiles;      // [num_tiles]
  const int* rowseq;      // [R] sequence of each row
  const int* seq_start;   // [n]
  const int* seq_len;     // [n]
  int num_tiles;
  int window;             // < 0: global
  int* err;
  unsigned long long wait_limit_ns;
  int stuck;
};
cudaError_t launch_attention_short(const CUtensorMap* tm_qkv, const AttnShortArgs& a, int num_sms,
                                   cudaStream_t stream);

// Longer sequences: tcgen05 flash attention (persistent, min(16 * items, num_sms) CTAs); tm_qkv
// maps the qkv buffer ([R, 3072] f16, box 64 columns x kAttnTcBoxRows rows,
// 128-byte swizzle): q at columns h*64, k at 1024 + h*64, v at 2048 + h*64.
cudaError_t launch_attention_tc(const CUtensorMap* tm_qkv, const AttnArgs& a, int num_sms, cudaStream_t stream);

// ---- row kernels -----------------------------------------------------------------
// x[r] = t[r] = LN(emb[tok[r]]) * w ; writes f32 residual and f16 copy
cudaError_t launch_embed_ln(const __half* emb, const int* tok, const float* w, float eps,
                            float* x, __half* t16, int rows, cudaStream_t s);
// t16[r] = LN(x[src(r)]) * w (+ b); src(r) = idx ? idx[r] : r
cudaError_t launch_ln(const float* x, const int* idx, const float* w, const float* b, float eps,
                      __half* t16, int rows, cudaStream_t s);
// x[r] = t16[r] = LN(x[r]) * w  (each warp reads its row before writing it)
cudaError_t launch_ln_inplace(float* x, const float* w, float eps, __half* t16, int rows, cudaStream_t s);
// Split-K partial sums waiting to be added to the residual stream: rows r >=
// row0 have them, part s of row r at parts[s * stride + (r - row0) * 1024 +
// c], s < nparts; rows below row0 have none.
struct PendingParts {
  const float* parts = nullptr;
  int nparts = 0;
  size_t stride = 0;
  int row0 = 0;
};
// x[r] += sum_s parts[s][r] (parts summed in order, then added);
// t16[r] = LN(x[r]) * w (+ b)
cudaError_t launch_ln_parts(float* x, const PendingParts& p, const float* w, const float* b, float eps,
                            __half* t16, int rows, cudaStream_t s);
// x[r] += sum_s parts[s][r] (the same arithmetic as launch_ln_parts)
cudaError_t launch_add_parts(float* x, const PendingParts& p, int rows, cudaStream_t s);
// x[r] = LN(x[r] (+ pending parts)) * wf + type[rowtype[r]];
// t16[r] = LN(x[r]) * w1 + b1
cudaError_t launch_final_ln(float* x, const float* wf, const __half* type_emb,
                            const uint8_t* rowtype, const float* w1, const float* b1,
                            float eps, __half* t16, int rows, cudaStream_t s,
                            const PendingParts& pend = PendingParts());

// ---- tail: scorer sum, post, act head --------------------------------------------
struct TailArgs {
  const float* partial;   // [kScorerPartials][ldp] scorer partial sums
  int ldp;
  float score_bias;
  const int8_t* mmask;    // [n*k]
  const int* cls_row;     // [n]
  const float* x;         // [R, 1024] residual stream after the head layers
  const __half* w1;       // [256, 1028]
  const float* b1;        // [256]
  const float* w2;        // [2, 256]
  const float* b2;        // [2]
  float* logits;          // [n*k]
  float* act;             // [n*2]
  int n, k;
};
cudaError_t launch_tail(const TailArgs& a, cudaStream_t s);

// Device pointers of the decision-tail weights an engine holds (scorer
// LayerNorm, scorer hidden projection and its tensor map, scorer output,
// act head), for launch paths outside the engine's own forward.
struct TailWeights {
  const float* ln_w;
  const float* ln_b;
  const CUtensorMap* hid_tmap;
  const float* hid_b;
  const float* wout;
  float bout;
  const __half* w1;
  const float* b1;
  const float* w2;
  const float* b2;
  int device;
  int num_sms;
};

}  // namespace laya
