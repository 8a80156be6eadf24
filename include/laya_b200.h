/*
 * laya_b200.h -- C ABI of the B200 (sm_100a) backend for the laya encoder
 * forward pass.
 *
 * The boundary is the reference's coarse engine seam (zerodegress/laya-rust):
 *   trait Engine { fn info(&self) -> EngineInfo; fn forward(&mut self, &Req) -> Out; }
 * (src/engine.rs:79-82) with Req (src/engine.rs:1-10) and Out
 * (src/engine.rs:12-17).  A Rust `CudaEngine` shim replacing
 * src/backend/cuda/mod.rs binds the functions below.
 *
 * Conventions
 *   - Every function returns LAYA_OK (0) or a nonzero status; the message of
 *     the calling thread's last failure is laya_last_error().  Nothing aborts
 *     the process (the reference panics; the shim maps status -> panic!).
 *   - Plain pointers and sizes only.  Host arrays are borrowed for the call.
 *   - One engine per GPU; an engine is used by one thread at a time
 *     (the reference's Engine takes &mut self and is not Sync).
 */
#ifndef LAYA_B200_H
#define LAYA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LAYA_OK = 0,
  LAYA_E_INVALID = 1,        /* malformed request or argument            */
  LAYA_E_LOAD = 2,           /* GGUF / weight validation failure         */
  LAYA_E_CUDA = 3,           /* CUDA runtime error                       */
  LAYA_E_DEVICE_TIMEOUT = 4, /* a bounded device-side wait expired       */
  LAYA_E_STATE = 5           /* call not valid in the engine's state     */
};

typedef struct laya_engine laya_engine;
typedef struct laya_plan laya_plan;

/* engine::Req (src/engine.rs:1-10).  ids/att are [n*l], mpos/mmask [n*k],
 * qtype [n]; att is 1 for real tokens and 0 for padding. */
typedef struct {
  int64_t n, l, k;
  const int64_t *ids;
  const int64_t *att;
  const int64_t *mpos;
  const int64_t *mmask;
  const int64_t *qtype;
} laya_req;

/* Message of the calling thread's most recent failure ("" if none). */
const char *laya_last_error(void);

/* Opens an engine on `device` and loads every weight from a GGUF v3 file,
 * validating metadata and shapes as Tensors::open does
 * (src/weights.rs:138-222, 233-245, 353-395).  Replaces CudaEngine::load
 * (src/backend/cuda/mod.rs:82-148). */
int laya_open(int device, const char *gguf_path, laya_engine **out);

/* Opens an engine with no weights, for a host that keeps its own GGUF loader
 * (the reference's gguf.rs / weights.rs): upload each of the 207 tensors with
 * laya_upload_weight_*, then laya_finalize. */
int laya_open_empty(int device, laya_engine **out);

/* Uploads one tensor named as in src/arch.rs, in STORED layout (the GGUF /
 * PyTorch [out, in] layout, dims as Tensors::stored_dims reports them,
 * src/weights.rs:261-268) -- not the transposed graph layout.  The copy is
 * complete on return; an upload that replaces a tensor first waits for the
 * engine's queued work (plan runs) that may still read the old one. */
int laya_upload_weight_f16(laya_engine *e, const char *name, const uint16_t *data,
                           const int64_t *stored_dims, int ndims);
int laya_upload_weight_f32(laya_engine *e, const char *name, const float *data,
                           const int64_t *stored_dims, int ndims);
/* Uploads one tensor exactly as the reference's unchanged loader hands it
 * out: the values of Tensors::f32 with the dims of Tensors::dims
 * (src/weights.rs:270-295), i.e. GRAPH layout, where the 120 matmul weights
 * of arch::transpose_names (src/arch.rs:306-322) are transposed to [in, out].
 * The engine transposes those back to the stored layout.  This is what the
 * reference's CudaEngine::load uploads (src/backend/cuda/mod.rs:125-132), so
 * a Rust shim can keep that loop unchanged. */
int laya_upload_weight_f32_graph(laya_engine *e, const char *name, const float *data,
                                 const int64_t *dims, int ndims);
/* Checks that all 207 tensors are present. */
int laya_finalize(laya_engine *e);

/* Engine::forward (src/engine.rs:81; CudaEngine::forward,
 * src/backend/cuda/mod.rs:466-812).  logits: n*k floats, act: n*2 floats,
 * host memory, written before return.  Requests must have att in prefix form
 * (ones then zeros in every row, at least one real token), qtype < 3,
 * 0 <= mpos < l, and mpos inside the real tokens where mmask != 0 -- the
 * layout build_batch produces (src/main.rs:470-500).
 * The engine keeps CUDA graphs of recent request shapes (batch shape, row
 * groups, attention work, arena generation; up to 8, least recently used
 * out): a shape's first call launches eagerly, its second is captured on the
 * engine's stream and later calls replay the graph, with the request uploaded
 * anew each call.  Results are bitwise those of the eager launch.  Weight
 * uploads and arena growth retire every graph.  One engine is not safe for
 * concurrent calls from several threads (neither is the reference's
 * &mut Engine).  LAYA_FORWARD_GRAPHS=0 in the environment disables the graphs. */
int laya_forward(laya_engine *e, const laya_req *req, float *logits, float *act);

/* TapSink (src/ops.rs:1-3): like laya_forward, and also calls fn with the
 * stages enc.{i}, final, head.{i}, logits, act.  Row stages are [n*l, 1024]
 * f32 in padded layout with zeros in padded rows.  Diagnostic path (slow). */
typedef void (*laya_tap_fn)(void *user, const char *stage, const float *data, size_t count);
int laya_forward_tapped(laya_engine *e, const laya_req *req, float *logits, float *act,
                        laya_tap_fn fn, void *user);

/* EngineInfo (src/engine.rs:71-77) as a JSON object in buf. */
int laya_info(laya_engine *e, char *buf, size_t len);
void laya_close(laya_engine *e);

/* ---- device-resident execution (no counterpart in the reference) -------------
 * A plan is a validated request uploaded once to device memory; running it
 * enqueues the forward on the engine's stream without host copies, so the
 * kernels can be timed with inputs resident in HBM. */
int laya_plan_create(laya_engine *e, const laya_req *req, laya_plan **out);
int laya_plan_run(laya_engine *e, laya_plan *p);
/* Synchronizes the stream, checks the device error word, copies outputs. */
int laya_plan_outputs(laya_engine *e, laya_plan *p, float *logits, float *act);
/* Captures the plan's launches into a CUDA graph; later runs replay it. */
int laya_plan_capture(laya_engine *e, laya_plan *p);
/* real_tokens: sum of real lengths; launches: kernels one run enqueues;
 * upload_bytes: bytes laya_forward copies host -> device for this request. */
int laya_plan_stats(laya_plan *p, int64_t *real_tokens, int64_t *launches, int64_t *upload_bytes);
/* Runs the plan `steps` times with a CUDA event recorded after every launch
 * and sums device time per launch kind into ms[LAYA_PROF_KINDS] and the
 * launch counts into launches[LAYA_PROF_KINDS].  Kinds: 0 GEMM QKV (encoder),
 * 1 GEMM attention-out, 2 GEMM FFN-in + GeGLU, 3 GEMM FFN-out, 4 GEMM head
 * layers and scorer, 5 attention, 6 row norms, 7 tail. */
#define LAYA_PROF_KINDS 8
int laya_plan_profile(laya_engine *e, laya_plan *p, int steps, double *ms, int64_t *launches);
void laya_plan_destroy(laya_plan *p);
/* The host side of a request's plan, with no device or engine (tests and
 * diagnostics): the validation laya_forward applies, with the same errors,
 * then the work the forward would launch.  *rows: the real tokens, compacted
 * sequence after sequence.  Tiles (2 ints each): (first row, rows) of the
 * attention tiles that pack consecutive sequences of at most 128 tokens.
 * Items (4 ints each): (first query row, query rows, sequence's first row,
 * sequence length) of the flash work items, one per 128 query rows of each
 * longer sequence, longest sequences first.  Counts are always written;
 * `tiles` / `items` may be NULL, else must hold cap_tiles / cap_items
 * entries (fewer than needed: LAYA_E_INVALID). */
int laya_plan_layout(const laya_req *req, int64_t *rows, int64_t *ntiles, int32_t *tiles, int64_t cap_tiles,
                     int64_t *nitems, int32_t *items, int64_t cap_items);
/* The cudaStream_t the engine launches on.  It is a non-blocking stream: work
 * the host issues on the legacy default stream (cudaMemcpy, cudaMemset, NULL-
 * stream launches) is not ordered with it, so a host that feeds or reads the
 * engine's buffers does so on this stream or synchronizes both. */
void *laya_stream(laya_engine *e);
/* One encoder layer in isolation (a benchmark configuration, the body of the
 * layer loop of graph.rs:103-123): set the residual stream of the plan's real
 * tokens (x: [real_tokens, 1024] f32, sequences back to back), enqueue layer
 * `layer` (0..27: input LN, QKV + RoPE, attention, Wo + residual, mlp_norm
 * LN, Wi + GeGLU, Wo_mlp + residual) on it, and read it back.  Layer 0's input
 * LN is the embedding norm and its residual base is the normed input
 * (graph.rs:112-113), so for layer 0 x is the embedding output.  Global layers
 * are the multiples of 3. */
int laya_plan_set_hidden(laya_engine *e, laya_plan *p, const float *x);
int laya_plan_run_layer(laya_engine *e, laya_plan *p, int layer);
int laya_plan_hidden(laya_engine *e, laya_plan *p, float *x);

/* ---- decision tail without allocation (no counterpart in the reference) -----
 * For hosts that cannot call cudaMalloc/cudaFree when they score: a serving
 * process whose device memory belongs to another allocator's pool, or a
 * latency-critical loop that cannot take an allocation's device sync.
 * Runs the scorer (LayerNorm over the gathered marker rows, 1024x1024 + bias,
 * GELU, 1024 -> 1 + bias), the marker post-processing and the act head -- the
 * same kernels the forward ends with -- on the caller's device buffers:
 *   x        f32 [rows, 1024]  final hidden rows (after the head layers)
 *   cls_row  int32 [n]         row of each sequence's first token
 *   mk_row   int32 [n*k]       row of each marker (any valid row if masked)
 *   mmask    int8  [n*k]       nonzero for real markers
 *   logits   f32 [n*k], act f32 [n*2]   outputs
 * Its scratch is one static device array sized for n*k <= 2048 rows (about
 * 4 MiB, resident on every GPU that loads the library); larger calls return
 * LAYA_E_INVALID.  No device memory is allocated by the call.  All calls share
 * that array: calls that overlap on the GPU race, so serialize them.  The
 * first call on a device (and with an engine) does set-up; make it before
 * any stream capture.  Set-up belongs to the device's primary context: a call
 * after the context was reset (cudaDeviceReset) finds the array's new address
 * and redoes it.  The engine's weight pointers are looked up again after any
 * weight upload.  The call runs on the engine's device and restores the
 * caller's current device before it returns.  Enqueues on `stream` (a
 * cudaStream_t, NULL for the default stream) and returns after synchronizing
 * it. */
#define LAYA_TAIL_STATIC_MAX_ROWS 2048
int laya_decision_tail_static(laya_engine *e, const float *x, int n, int k, const int32_t *cls_row,
                              const int32_t *mk_row, const int8_t *mmask, float *logits, float *act,
                              void *stream);

/* ---- kernel self-tests (no counterpart in the reference) --------------------
 * Host in, host out; used by the GPU tests to check single kernels. */
/* out[M,N] (f32) = A[M,K] . W[N,K]^T with A, W f16, on 256 x tile_n tiles
 * (tile_n 256 or 128); N % tile_n == 0, K % 64 == 0. */
int laya_selftest_gemm(int device, const uint16_t *a, const uint16_t *w, float *out, int m,
                       int n, int k, int tile_n);
/* Times the GEMM alone with one of the forward's epilogues: f16 operands of
 * a fixed pattern on the device, `iters` launches of epi(A[M,K] . W[N,K]^T)
 * on 256 x tile_n tiles, each bracketed by CUDA events; with flush_l2 != 0 a
 * 256 MiB memset runs (untimed) before every launch so operands start cold.
 * epi: 0 QKV + RoPE (n = 3072, f16 out), 1 QKV + bias, 2 residual add into
 * f32 [M,N], 3 GeGLU (n = gate/up co-tiled columns, f16 out [M, n/2]),
 * 4 bias + ReLU, 6 f32 store; tile_n 128 only for 2 and 6.
 * *ms = mean device time per launch. */
int laya_bench_gemm(int device, int m, int n, int k, int tile_n, int epi, int flush_l2, int iters, float *ms);

/* Test of the device-side bounded waits (failure detection without a GPU
 * fault): arms the engine so that in its next forward
 * (or plan run) the first launch of `kind` (0: the first GEMM, 1: the first
 * attention launch) makes its TMA producers wait, before issuing any load, on
 * an mbarrier that nothing ever completes, bounded by `limit_ns` (at most 2 s).
 * The wait expires, the kernel records the error, unwinds and returns; the
 * forward then reports LAYA_E_DEVICE_TIMEOUT and the engine stays usable.
 * One-shot: the forward after that one runs normally. */
int laya_test_timeout_next(laya_engine *e, int kind, uint64_t limit_ns);

/* Ragged attention on qkv [R,3072] f16 (q,k pre-scaled) for sequences packed
 * back to back with lengths lens[n]; window < 0 for global.  out [R,1024] f32.
 * impl must be 1 (the tcgen05 kernel the forward uses). */
int laya_selftest_attention(int device, const uint16_t *qkv, const int32_t *lens, int n,
                            int window, float *out, int impl);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_B200_H */
