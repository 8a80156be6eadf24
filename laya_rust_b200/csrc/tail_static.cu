// Decision tail that allocates no device memory.
//
// Same computation as the last three launches of the engine's forward
// (scorer LayerNorm over the gathered marker rows, the scorer GEMM with its
// GELU . w_out epilogue, then post + act head), but its scratch -- the gathered
// f16 marker rows and the per-tile scorer partial sums -- lives in one
// file-scope static device array instead of the engine's cudaMalloc'd arena.
//
// Who needs it: a host that cannot call cudaMalloc/cudaFree at the point where
// it scores, e.g. a serving process whose device memory is owned by another
// allocator's pool (a framework caching allocator that has reserved the GPU),
// or a latency-critical loop where an allocation's implicit device
// synchronisation is not acceptable.  The caller passes device pointers for
// every input and output; this file uses only the static array.
//
// Limits and sharing:
//   * at most kStaticMaxRows = n*k marker rows per call (larger calls are
//     rejected with LAYA_E_INVALID); the array (4 MiB of rows + 64 KiB of
//     partial sums + an error word) stays allocated on every GPU that loads
//     the library until the process exits;
//   * every call on a device shares the one array and it keeps the previous
//     call's contents; nothing in it needs to start at zero except the error
//     word, which each call clears.  Calls whose work overlaps on the GPU
//     (two streams, or two host threads) race on the array: serialize them;
//   * every call looks up the array's device address with
//     cudaGetSymbolAddress on the engine's device (host code cannot use the
//     symbol itself: in host code it names a host-side shadow, not device
//     memory).  The first call on a device, and any call after the address
//     changed (a new primary context, e.g. after cudaDeviceReset), encodes the
//     TMA tensor map over it.  The engine's weight pointers are cached until
//     a weight is uploaded again.  Make the first call before any stream
//     capture;
//   * the call switches to the engine's device and restores the caller's
//     current device before it returns.
#include <mutex>

#include "../../include/laya_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace laya {

bool engine_tail_weights(laya_engine* e, TailWeights* out, int* status);
void set_last_error(const char* msg);

namespace {

constexpr int kStaticMaxRows = LAYA_TAIL_STATIC_MAX_ROWS;
constexpr int kHid = 1024;
constexpr size_t kRowsBytes = static_cast<size_t>(kStaticMaxRows) * kHid * sizeof(__half);
constexpr size_t kPartialBytes = static_cast<size_t>(kScorerPartials) * kStaticMaxRows * sizeof(float);
constexpr size_t kScratchBytes = kRowsBytes + kPartialBytes + 256;

// [rows f16 | partial f32 | error word]
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

struct DeviceState {
  bool ready = false;
  unsigned char* base = nullptr;  // device address of g_scratch on this device
  CUtensorMap rows_map;
};

DeviceState g_state[64];
std::mutex g_mu;

// With device `dev` current: resolve the array's device address and, when it
// is new (first call on the device, or a new primary context since), build
// the tensor map the scorer GEMM reads it through.
int setup_device(int dev, DeviceState** out) {
  if (dev < 0 || dev >= 64) {
    set_last_error("decision_tail_static: device index out of range");
    return LAYA_E_INVALID;
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_last_error(cudaGetErrorString(e));
    return LAYA_E_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& s = g_state[dev];
  if (!s.ready || s.base != p) {
    s.ready = false;
    s.base = static_cast<unsigned char*>(p);
    if (make_tmap_f16(&s.rows_map, s.base, kStaticMaxRows, kHid, kGemmABoxRows) != 0) {
      set_last_error("decision_tail_static: tensor map encode failed");
      return LAYA_E_CUDA;
    }
    s.ready = true;
  }
  *out = &s;
  return LAYA_OK;
}

// Restores the caller's current device when the call returns.
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  }
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int fail(cudaError_t e) {
  set_last_error(cudaGetErrorString(e));
  return LAYA_E_CUDA;
}

}  // namespace
}  // namespace laya

extern "C" int laya_decision_tail_static(laya_engine* e, const float* x, int n, int k, const int32_t* cls_row,
                                         const int32_t* mk_row, const int8_t* mmask, float* logits, float* act,
                                         void* stream) {
  using namespace laya;
  if (!e || !x || !cls_row || !mk_row || !mmask || !logits || !act) {
    set_last_error("decision_tail_static: null argument");
    return LAYA_E_INVALID;
  }
  if (n <= 0 || k <= 0 || static_cast<long long>(n) * k > kStaticMaxRows) {
    set_last_error("decision_tail_static: n*k must be in [1, LAYA_TAIL_STATIC_MAX_ROWS]");
    return LAYA_E_INVALID;
  }
  TailWeights w;
  int status = LAYA_OK;
  if (!engine_tail_weights(e, &w, &status)) return status;
  DeviceRestore restore;
  cudaError_t ce = cudaSetDevice(w.device);
  if (ce != cudaSuccess) return fail(ce);
  DeviceState* s = nullptr;
  status = setup_device(w.device, &s);
  if (status != LAYA_OK) return status;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* rows = reinterpret_cast<__half*>(s->base);
  float* partial = reinterpret_cast<float*>(s->base + kRowsBytes);
  int* err = reinterpret_cast<int*>(s->base + kRowsBytes + kPartialBytes);
  const int nk = n * k;

  if ((ce = cudaMemsetAsync(err, 0, sizeof(int), st)) != cudaSuccess) return fail(ce);
  if ((ce = launch_ln(x, mk_row, w.ln_w, w.ln_b, 1e-5f, rows, nk, st)) != cudaSuccess) return fail(ce);
  GemmArgs g{};
  g.M = nk;
  g.N = kHid;
  g.K = kHid;
  g.err = err;
  g.out = partial;
  g.ldo = kStaticMaxRows;
  g.bias = w.hid_b;
  g.wvec = w.wout;
  if ((ce = launch_gemm(kEpiScorer, GemmMaps{&s->rows_map, w.hid_tmap, &s->rows_map}, g, w.num_sms, st)) !=
      cudaSuccess)
    return fail(ce);
  TailArgs t{};
  t.partial = partial;
  t.ldp = kStaticMaxRows;
  t.score_bias = w.bout;
  t.mmask = mmask;
  t.cls_row = cls_row;
  t.x = x;
  t.w1 = w.w1;
  t.b1 = w.b1;
  t.w2 = w.w2;
  t.b2 = w.b2;
  t.logits = logits;
  t.act = act;
  t.n = n;
  t.k = k;
  if ((ce = launch_tail(t, st)) != cudaSuccess) return fail(ce);
  int dev_err = 0;
  if ((ce = cudaMemcpyAsync(&dev_err, err, sizeof(int), cudaMemcpyDeviceToHost, st)) != cudaSuccess) return fail(ce);
  if ((ce = cudaStreamSynchronize(st)) != cudaSuccess) return fail(ce);
  if (dev_err != 0) {
    set_last_error("decision_tail_static: a device-side wait expired");
    return LAYA_E_DEVICE_TIMEOUT;
  }
  set_last_error("");
  return LAYA_OK;
}
