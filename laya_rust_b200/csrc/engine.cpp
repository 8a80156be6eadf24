// Host engine behind the C ABI (include/laya_b200.h).
//
// Replaces laya-rust's CudaEngine (src/backend/cuda/mod.rs): weight residency,
// buffer arena, per-request upload and the launch sequence of the forward.
// The graph it runs is graph.rs:86-186; the weight roles and stored shapes are
// arch.rs:263-322 and weights.rs:353-395; metadata checks weights.rs:138-222.
//
// Differences from the reference, by design:
//   * weights stay f16 as stored ([out, in], K-major), no widening and no host
//     transposes (the reference widens to f32 and transposes 120 tensors);
//   * the forward runs on the real tokens only: each row's att prefix is
//     compacted into one token-major buffer (cu_seqlens layout), the padded
//     positions are never computed (their outputs never reach logits/act);
//   * no mask tensor: attention takes (length, window) predicates.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/laya_b200.h"
#include "gguf_reader.h"
#include "kernels.h"

namespace laya {

// ---- constants (arch.rs:1-15) -------------------------------------------------------
constexpr int H = 1024, NH = 16, HD = 64, NLAYER = 28, INTER = 2624, NVOCAB = 50368;
constexpr float SCALE = 0.3535533845424652f, EPS = 1e-5f;
constexpr int WINDOW = 64, HEAD_LAYERS = 2, HEAD_INTER = 4096, ACT_HIDDEN = 256, ACT_INPUT = H + 4;
constexpr int QTYPES = 3, GLOBAL_EVERY = 3;
constexpr int INTER_PAD = 2688;  // 21 tiles of 128 gate columns (2624 rounded up)

namespace {

thread_local std::string g_err;

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(LAYA_E_CUDA, fmt("%s: %s", what, cudaGetErrorString(e)));
}

template <class F>
int guard(F&& f) {
  try {
    f();
    g_err.clear();
    return LAYA_OK;
  } catch (const Error& e) {
    g_err = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_err = "out of host memory";
    return LAYA_E_INVALID;
  } catch (const std::exception& e) {
    g_err = e.what();
    return LAYA_E_LOAD;
  }
}

uint16_t f2h_bits(float f) {
  __half h = __float2half_rn(f);
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

float h2f_bits(uint16_t b) {
  __half_raw r;
  r.x = b;
  return __half2float(__half(r));
}

// ---- weight roles ---------------------------------------------------------------------
enum class Kind { Linear, Embed, F32Vec, F32Mat, Rope, ActW1 };

struct Role {
  Kind kind;
  std::vector<int64_t> shape;  // stored shape (weights.rs:353-395)
};

std::string attn_norm(int i) {
  return i == 0 ? "encoder.embeddings.norm.weight" : fmt("encoder.layers.%d.attn_norm.weight", i);
}

std::map<std::string, Role> build_roles() {
  std::map<std::string, Role> r;
  r["encoder.embeddings.tok_embeddings.weight"] = {Kind::Embed, {NVOCAB, H}};
  r["type_emb.weight"] = {Kind::Embed, {QTYPES, H}};
  r["encoder.final_norm.weight"] = {Kind::F32Vec, {H}};
  r["rope.freq_full"] = {Kind::Rope, {HD / 2}};
  r["rope.freq_sliding"] = {Kind::Rope, {HD / 2}};
  r["scorer.0.weight"] = {Kind::F32Vec, {H}};
  r["scorer.0.bias"] = {Kind::F32Vec, {H}};
  r["scorer.1.weight"] = {Kind::Linear, {H, H}};
  r["scorer.1.bias"] = {Kind::F32Vec, {H}};
  r["scorer.3.weight"] = {Kind::F32Mat, {1, H}};
  r["scorer.3.bias"] = {Kind::F32Vec, {1}};
  r["act_head.0.weight"] = {Kind::ActW1, {ACT_HIDDEN, ACT_INPUT}};
  r["act_head.0.bias"] = {Kind::F32Vec, {ACT_HIDDEN}};
  r["act_head.2.weight"] = {Kind::F32Mat, {2, ACT_HIDDEN}};
  r["act_head.2.bias"] = {Kind::F32Vec, {2}};
  for (int i = 0; i < NLAYER; ++i) {
    r[attn_norm(i)] = {Kind::F32Vec, {H}};
    r[fmt("encoder.layers.%d.mlp_norm.weight", i)] = {Kind::F32Vec, {H}};
    r[fmt("encoder.layers.%d.attn.Wqkv.weight", i)] = {Kind::Linear, {3 * H, H}};
    r[fmt("encoder.layers.%d.attn.Wo.weight", i)] = {Kind::Linear, {H, H}};
    r[fmt("encoder.layers.%d.mlp.Wi.weight", i)] = {Kind::Linear, {2 * INTER, H}};
    r[fmt("encoder.layers.%d.mlp.Wo.weight", i)] = {Kind::Linear, {H, INTER}};
  }
  for (int i = 0; i < HEAD_LAYERS; ++i) {
    auto n = [&](const char* s) { return fmt("head.layers.%d.%s", i, s); };
    r[n("norm1.weight")] = {Kind::F32Vec, {H}};
    r[n("norm1.bias")] = {Kind::F32Vec, {H}};
    r[n("norm2.weight")] = {Kind::F32Vec, {H}};
    r[n("norm2.bias")] = {Kind::F32Vec, {H}};
    r[n("self_attn.in_proj_weight")] = {Kind::Linear, {3 * H, H}};
    r[n("self_attn.in_proj_bias")] = {Kind::F32Vec, {3 * H}};
    r[n("self_attn.out_proj.weight")] = {Kind::Linear, {H, H}};
    r[n("self_attn.out_proj.bias")] = {Kind::F32Vec, {H}};
    r[n("linear1.weight")] = {Kind::Linear, {HEAD_INTER, H}};
    r[n("linear1.bias")] = {Kind::F32Vec, {HEAD_INTER}};
    r[n("linear2.weight")] = {Kind::Linear, {H, HEAD_INTER}};
    r[n("linear2.bias")] = {Kind::F32Vec, {H}};
  }
  return r;
}

// The 120 weights Tensors::f32 transposes to graph layout (arch.rs:306-322):
// every encoder layer's Wqkv, Wo, Wi and mlp.Wo, the head layers' in_proj,
// linear1 and linear2, and the scorer's two linear weights.
bool in_transpose_set(const std::string& name) {
  static const std::set<std::string> names = [] {
    std::set<std::string> s;
    for (int i = 0; i < NLAYER; ++i)
      for (const char* w : {"attn.Wqkv.weight", "attn.Wo.weight", "mlp.Wi.weight", "mlp.Wo.weight"})
        s.insert(fmt("encoder.layers.%d.%s", i, w));
    for (int i = 0; i < HEAD_LAYERS; ++i)
      for (const char* w : {"self_attn.in_proj_weight", "linear1.weight", "linear2.weight"})
        s.insert(fmt("head.layers.%d.%s", i, w));
    s.insert("scorer.1.weight");
    s.insert("scorer.3.weight");
    return s;
  }();
  return names.count(name) > 0;
}

const std::map<std::string, Role>& roles() {
  static const std::map<std::string, Role> r = build_roles();
  return r;
}

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  void alloc(size_t b, const char* what) {
    release();
    ck(cudaMalloc(&p, b), what);
    bytes = b;
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct Weight {
  DevBuf buf;
  CUtensorMap tmap;         // Linear weights only
  CUtensorMap tmap_narrow;  // Linear weights: box for 256 x 128 tiles (small batches)
  std::vector<float> host;  // small tensors the host also needs (rope, scorer bias)
  bool present = false;
};

// Host-side plan of one request: validated and compacted (real tokens only).
// Rows [row0, row0 + rows) of the compacted batch (whole sequences) whose
// encoder and head layers run as one chain of launches; its attention work
// is tiles[tile0, tile0 + ntiles) (packed sequences of at most kAttnTcQRows
// tokens) and items[item0, item0 + nitems) (128-row blocks of longer ones).
struct RowGroup {
  int row0 = 0, rows = 0, tile0 = 0, ntiles = 0, item0 = 0, nitems = 0;
};

// With LAYA_ROW_GROUPS=2, batches of at least kSplitMinRows real tokens run as
// two row groups on two streams, so that one group's kernels can fill the SMs
// the other's leave idle (a GEMM's last partial wave, launch gaps, row-norm
// and attention tails).  Off by default: measured on the 16384-token forward
// it is 1% slower (9.45 vs 9.37 ms), since the persistent GEMM assigns tiles
// statically and a cluster that starts late behind the other stream's kernel
// still owns its full share.
constexpr int kSplitMinRows = 2048;

bool row_groups_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_ROW_GROUPS");
    return v && v[0] == '2';
  }();
  return on;
}

// Split-K for the residual GEMMs (Wo, Wo_mlp) of small batches: when the
// 256 x 256 output tiles fill at most half the clusters, the K loop is cut
// into parts that run on otherwise idle SMs; each part stores its f32 sums
// (kEpiPartial) and the LayerNorm that follows adds them to the residual in
// part order, so results stay bitwise reproducible.  LAYA_SPLITK=0 turns it
// off.  kPartRows bounds parts x padded rows over every M the rule admits
// (at most 4608: e.g. 9 row blocks x 2 parts, 3 x 6).
constexpr int kPartRows = 4608;

// The public forward replays a CUDA graph per request shape (captured on
// the shape's second call); LAYA_FORWARD_GRAPHS=0 launches every forward
// eagerly.  At most kForwardGraphs shapes are kept (least recently used out).
constexpr size_t kForwardGraphs = 8;
bool forward_graphs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_FORWARD_GRAPHS");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Narrow (256 x 128) tiles for the f16-output GEMMs of small batches;
// LAYA_NARROW=0 keeps 256 x 256 tiles everywhere.
bool narrow_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_NARROW");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool splitk_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_SPLITK");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Large batches: a residual GEMM whose 256 x 256 tiles leave the last wave at
// most half full splits the K loop of its last row blocks instead, so the
// last wave is short (kEpiResidTail).  LAYA_TAILSPLIT=0 turns it off.
bool tailsplit_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_TAILSPLIT");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Most K parts per GEMM (LAYA_SPLITK_MAX, 2..8; default 4: on the 179-token
// request 4 and 8 parts measured the same, 1.98 ms, and 4 reads half the
// parts back).
int splitk_max() {
  static const int n = [] {
    const char* v = std::getenv("LAYA_SPLITK_MAX");
    const int k = v ? std::atoi(v) : 4;
    return k < 2 ? 2 : (k > 8 ? 8 : k);
  }();
  return n;
}

struct HostPlan {
  int n = 0, l = 0, k = 0, R = 0, ntiles = 0, nitems = 0;
  std::vector<int> tok, pos, seq_start, seq_len, cls_row, mk_row, rowseq;
  // attention work per row group (see pack_short_tiles, attention_items)
  std::vector<int2> tiles;
  std::vector<int4> items;
  std::vector<RowGroup> groups;
  std::vector<uint8_t> rowtype;
  std::vector<int8_t> mmask;
};

// Offsets of each array inside one packed device buffer.
struct PlanLayout {
  size_t tok, pos, seq_start, seq_len, cls_row, mk_row, tiles, items, rowtype, mmask, rowseq, total;
};

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

PlanLayout layout_for(const HostPlan& p) {
  PlanLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += up256(bytes ? bytes : 1);
    return at;
  };
  L.tok = take(sizeof(int) * p.R);
  L.pos = take(sizeof(int) * p.R);
  L.seq_start = take(sizeof(int) * p.n);
  L.seq_len = take(sizeof(int) * p.n);
  L.cls_row = take(sizeof(int) * p.n);
  L.mk_row = take(sizeof(int) * p.n * p.k);
  L.tiles = take(sizeof(int2) * p.ntiles);
  L.items = take(sizeof(int4) * p.nitems);
  L.rowtype = take(p.R);
  L.mmask = take((size_t)p.n * p.k);
  L.rowseq = take(sizeof(int) * p.R);
  L.total = o;
  return L;
}

void pack(const HostPlan& p, const PlanLayout& L, uint8_t* dst) {
  memcpy(dst + L.tok, p.tok.data(), sizeof(int) * p.R);
  memcpy(dst + L.pos, p.pos.data(), sizeof(int) * p.R);
  memcpy(dst + L.seq_start, p.seq_start.data(), sizeof(int) * p.n);
  memcpy(dst + L.seq_len, p.seq_len.data(), sizeof(int) * p.n);
  memcpy(dst + L.cls_row, p.cls_row.data(), sizeof(int) * p.n);
  memcpy(dst + L.mk_row, p.mk_row.data(), sizeof(int) * p.n * p.k);
  memcpy(dst + L.tiles, p.tiles.data(), sizeof(int2) * p.ntiles);
  memcpy(dst + L.items, p.items.data(), sizeof(int4) * p.nitems);
  memcpy(dst + L.rowtype, p.rowtype.data(), p.R);
  memcpy(dst + L.mmask, p.mmask.data(), (size_t)p.n * p.k);
  memcpy(dst + L.rowseq, p.rowseq.data(), sizeof(int) * p.R);
}

// Attention tiles for the sequences of at most kAttnTcQRows tokens among
// [b0, b1): consecutive ones (adjacent in the compacted rows) share a tile
// while their rows fit, as (first row, rows).
void pack_short_tiles(const std::vector<int>& start, const std::vector<int>& len, int b0, int b1,
                      std::vector<int2>& out) {
  int row0 = -1, rows = 0;
  for (int b = b0; b < b1; ++b) {
    if (len[b] > kAttnTcQRows) {
      if (row0 >= 0) out.push_back(make_int2(row0, rows));
      row0 = -1;
      continue;
    }
    if (row0 >= 0 && start[b] == row0 + rows && rows + len[b] <= kAttnTcQRows) {
      rows += len[b];
    } else {
      if (row0 >= 0) out.push_back(make_int2(row0, rows));
      row0 = start[b];
      rows = len[b];
    }
  }
  if (row0 >= 0) out.push_back(make_int2(row0, rows));
}

// Flash-attention work items for the sequences longer than kAttnTcQRows
// tokens among [b0, b1): int4 (first query row, query rows, sequence start
// row, sequence length), one per block of kAttnTcQRows query rows, longest
// sequences first (they see the most key blocks, so the persistent kernel's
// round-robin deals them out first; ties keep sequence order).
void attention_items(const std::vector<int>& start, const std::vector<int>& len, int b0, int b1,
                     std::vector<int4>& out) {
  std::vector<int> order;
  for (int b = b0; b < b1; ++b)
    if (len[b] > kAttnTcQRows) order.push_back(b);
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return len[x] > len[y]; });
  for (int b : order)
    for (int q0 = 0; q0 < len[b]; q0 += kAttnTcQRows)
      out.push_back(make_int4(start[b] + q0, std::min(kAttnTcQRows, len[b] - q0), start[b], len[b]));
}

// Validates a Req and compacts its real tokens.  The reference asserts
// n, l, k > 0 (graph.rs:93) and indexes ids / mpos / qtype unchecked
// (cpu/mod.rs:145-153, 372-398) -- out-of-range values panic there and are
// rejected here.
HostPlan make_plan(const laya_req* q) {
  if (!q) throw Error(LAYA_E_INVALID, "null request");
  if (q->n <= 0 || q->l <= 0 || q->k <= 0)
    throw Error(LAYA_E_INVALID, fmt("request needs n, l, k > 0 (got %lld, %lld, %lld)", (long long)q->n,
                                    (long long)q->l, (long long)q->k));
  if (!q->ids || !q->att || !q->mpos || !q->mmask || !q->qtype) throw Error(LAYA_E_INVALID, "null request array");
  if (q->n > (1 << 20) || q->l > (1 << 16) || q->k > 4096 || q->n * q->l > (1 << 24))
    throw Error(LAYA_E_INVALID, "request too large");
  HostPlan p;
  p.n = (int)q->n;
  p.l = (int)q->l;
  p.k = (int)q->k;
  p.seq_start.resize(p.n);
  p.seq_len.resize(p.n);
  int R = 0;
  for (int b = 0; b < p.n; ++b) {
    const int64_t* att = q->att + (size_t)b * p.l;
    int r = 0;
    while (r < p.l && att[r] != 0) ++r;
    for (int t = r; t < p.l; ++t)
      if (att[t] != 0)
        throw Error(LAYA_E_INVALID,
                    fmt("row %d: att is not a prefix of ones (real token at %d after padding at %d)", b, t, r));
    if (r == 0) throw Error(LAYA_E_INVALID, fmt("row %d has no real tokens", b));
    const int64_t qt = q->qtype[b];
    if (qt < 0 || qt >= QTYPES) throw Error(LAYA_E_INVALID, fmt("row %d: qtype %lld out of range", b, (long long)qt));
    p.seq_start[b] = R;
    p.seq_len[b] = r;
    R += r;
  }
  p.R = R;
  p.tok.resize(R);
  p.pos.resize(R);
  p.rowtype.resize(R);
  p.rowseq.resize(R);
  for (int b = 0; b < p.n; ++b) {
    const int64_t* ids = q->ids + (size_t)b * p.l;
    for (int t = 0; t < p.l; ++t)
      if (ids[t] < 0 || ids[t] >= NVOCAB)
        throw Error(LAYA_E_INVALID, fmt("row %d: token id %lld at %d out of range", b, (long long)ids[t], t));
    for (int t = 0; t < p.seq_len[b]; ++t) {
      p.tok[p.seq_start[b] + t] = (int)ids[t];
      p.pos[p.seq_start[b] + t] = t;
      p.rowtype[p.seq_start[b] + t] = (uint8_t)q->qtype[b];
      p.rowseq[p.seq_start[b] + t] = b;
    }
  }
  // two row groups of about R/2 rows, split at a sequence boundary
  int split = p.n;
  if (p.n >= 2 && R >= kSplitMinRows && row_groups_enabled()) {
    int best = R;
    for (int b = 1; b < p.n; ++b) {
      const int d = std::abs(2 * p.seq_start[b] - R);
      if (d < best) {
        best = d;
        split = b;
      }
    }
  }
  const int bounds[3] = {0, split, p.n};
  for (int gi = 0; gi < (split < p.n ? 2 : 1); ++gi) {
    RowGroup g;
    const int b0 = bounds[gi], b1 = bounds[gi + 1];
    g.row0 = p.seq_start[b0];
    g.rows = (b1 < p.n ? p.seq_start[b1] : R) - g.row0;
    g.tile0 = (int)p.tiles.size();
    pack_short_tiles(p.seq_start, p.seq_len, b0, b1, p.tiles);
    g.ntiles = (int)p.tiles.size() - g.tile0;
    g.item0 = (int)p.items.size();
    attention_items(p.seq_start, p.seq_len, b0, b1, p.items);
    g.nitems = (int)p.items.size() - g.item0;
    p.groups.push_back(g);
  }
  p.ntiles = (int)p.tiles.size();
  p.nitems = (int)p.items.size();
  p.cls_row.resize(p.n);
  p.mk_row.resize((size_t)p.n * p.k);
  p.mmask.resize((size_t)p.n * p.k);
  for (int b = 0; b < p.n; ++b) {
    p.cls_row[b] = p.seq_start[b];
    for (int j = 0; j < p.k; ++j) {
      const size_t i = (size_t)b * p.k + j;
      const int64_t mp = q->mpos[i];
      const bool on = q->mmask[i] != 0;
      if (mp < 0 || mp >= p.l)
        throw Error(LAYA_E_INVALID, fmt("marker %d of row %d: position %lld outside [0, %d)", j, b, (long long)mp, p.l));
      if (on && mp >= p.seq_len[b])
        throw Error(LAYA_E_INVALID, fmt("marker %d of row %d at %lld points at padding (real length %d)", j, b,
                                        (long long)mp, p.seq_len[b]));
      p.mmask[i] = on ? 1 : 0;
      // masked markers read the sequence's first row: their logit is
      // replaced by -10000 regardless of the score (cpu/mod.rs:409)
      p.mk_row[i] = p.seq_start[b] + (on ? (int)mp : 0);
    }
  }
  return p;
}

}  // namespace

// Tensor maps over the arena with this plan's exact row counts: TMA loads
// zero-fill rows past the last real token, TMA stores clip them.
struct GroupMaps {
  CUtensorMap a_t16, a_ctx, a_gate, a_hmlp;  // GEMM A operands over the group's rows
  CUtensorMap o_qkv, o_x, o_gate, o_hmlp;    // GEMM outputs over the group's rows
};

struct PlanMaps {
  GroupMaps g[2];
  CUtensorMap a_mk;                                // scorer A operand (gathered marker rows)
  CUtensorMap qkv_rows;                            // attention: 64-column x 32-row boxes of qkv
  uint64_t gen = ~0ull;                            // arena generation encoded for
};

struct DevicePlan {
  HostPlan host;
  PlanLayout lay;
  PlanMaps maps;
  DevBuf own;              // the plan's own device copy (laya_plan_create)
  uint8_t* base = nullptr; // where the packed arrays live (own, or the engine's buffer)
  cudaGraphExec_t graph = nullptr;
  uint64_t graph_arena_gen = 0;
  int64_t launches = 0;
  ~DevicePlan() {
    if (graph) cudaGraphExecDestroy(graph);
  }
  template <class T>
  const T* at(size_t off) const {
    return reinterpret_cast<const T*>(base + off);
  }
};

struct Engine {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  cudaStream_t side = nullptr;  // second row group's stream
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  std::string device_name;
  std::map<std::string, Weight> w;
  float temperature[3] = {1, 1, 1};
  std::string temperature_by_options = "{}";
  int file_type = 1;
  bool finalized = false;

  // rope tables [rope_len][32] for the full (global) and sliding frequencies
  DevBuf cos_full, sin_full, cos_slide, sin_slide;
  int rope_len = 0;

  // arena
  int cap_rows = 0, cap_mk = 0, cap_n = 0;
  // bumped on every arena reallocation and weight upload; captured graphs and
  // plan tensor maps record it
  uint64_t arena_gen = 0;
  DevBuf x, t16, qkv, ctx, gate, hmlp, mk16, partial, out_logits, out_act, err, plan_buf;
  // split-K parts of the residual GEMMs, one region per row group, and the
  // parts each group's next LayerNorm still has to add
  DevBuf parts[2];
  CUtensorMap parts_map[2];
  bool parts_ready = false;
  PendingParts pend[2];
  uint8_t* staging = nullptr;    // pinned host staging for plan uploads
  size_t staging_bytes = 0;
  float* pinned_out = nullptr;   // pinned staging for outputs
  size_t pinned_out_floats = 0;

  // launch profiling (laya_plan_profile): an event after every launch
  enum ProfKind { kProfQkv, kProfWo, kProfWi, kProfWo2, kProfHead, kProfAttn, kProfNorm, kProfTail };
  std::vector<cudaEvent_t>* prof_ev = nullptr;
  std::vector<int>* prof_kind = nullptr;

  // The timeout test (laya_test_timeout_next): the next forward's first
  // launch of the chosen kind waits on a barrier nothing completes, with
  // this limit, so that its device-side wait expires and the kernel unwinds.
  bool stuck_next = false;
  int stuck_kind = 0;  // 0: the first GEMM, 1: the first attention launch
  unsigned long long stuck_limit_ns = 0;

  // decision-tail weight pointers, looked up once (see tail_weights)
  TailWeights tail_cache{};
  bool tail_cache_ready = false;

  const TailWeights& tail_weights() {
    if (!tail_cache_ready) {
      TailWeights t{};
      t.ln_w = W("scorer.0.weight").buf.as<float>();
      t.ln_b = W("scorer.0.bias").buf.as<float>();
      t.hid_tmap = &W("scorer.1.weight").tmap;
      t.hid_b = W("scorer.1.bias").buf.as<float>();
      t.wout = W("scorer.3.weight").buf.as<float>();
      t.bout = W("scorer.3.bias").host[0];
      t.w1 = W("act_head.0.weight").buf.as<__half>();
      t.b1 = W("act_head.0.bias").buf.as<float>();
      t.w2 = W("act_head.2.weight").buf.as<float>();
      t.b2 = W("act_head.2.bias").buf.as<float>();
      t.device = device;
      t.num_sms = num_sms;
      tail_cache = t;
      tail_cache_ready = true;
    }
    return tail_cache;
  }

  void mark(int kind) {
    if (!prof_ev) return;
    cudaEvent_t ev;
    ck(cudaEventCreate(&ev), "event create");
    prof_ev->push_back(ev);
    prof_kind->push_back(kind);
    ck(cudaEventRecord(ev, stream), "event record");
  }

  // CUDA graphs of the public forward, keyed by everything a launch's
  // arguments depend on (forward_graph_key); a shape is captured on its
  // second call and replayed from then on.  Entries of an older arena
  // generation (arena or RoPE tables moved, a weight uploaded) are dropped.
  struct FwdGraph {
    std::vector<int64_t> key;
    cudaGraphExec_t exec = nullptr;
    uint64_t gen = 0;
    uint64_t last_use = 0;
  };
  std::vector<FwdGraph> fwd_graphs;
  std::map<std::vector<int64_t>, int> fwd_seen;
  uint64_t fwd_clock = 0;

  void drop_forward_graphs() {
    for (auto& g : fwd_graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    fwd_graphs.clear();
    fwd_seen.clear();
  }

  ~Engine() {
    if (stream) cudaStreamSynchronize(stream);
    drop_forward_graphs();
    if (pinned_out) cudaFreeHost(pinned_out);
    if (staging) cudaFreeHost(staging);
    if (side) cudaStreamSynchronize(side);
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (side) cudaStreamDestroy(side);
    if (stream) cudaStreamDestroy(stream);
  }

  void set_device() { ck(cudaSetDevice(device), "cudaSetDevice"); }

  const Weight& W(const std::string& name) const {
    auto it = w.find(name);
    if (it == w.end() || !it->second.present) throw Error(LAYA_E_STATE, "weight " + name + " was not loaded");
    return it->second;
  }

  // ---- weights ------------------------------------------------------------------
  void upload(const std::string& name, const void* data, bool is_f16, const int64_t* dims, int nd) {
    auto it = roles().find(name);
    if (it == roles().end()) throw Error(LAYA_E_LOAD, "unknown tensor name " + name);
    const Role& role = it->second;
    std::vector<int64_t> got(dims, dims + nd);
    if (got != role.shape) {
      std::string g, e;
      for (auto d : got) g += std::to_string(d) + ",";
      for (auto d : role.shape) e += std::to_string(d) + ",";
      throw Error(LAYA_E_LOAD, "tensor " + name + " has stored shape [" + g + "] but this build pins [" + e + "]");
    }
    size_t el = 1;
    for (auto d : got) el *= (size_t)d;
    auto f32_at = [&](size_t i) {
      return is_f16 ? h2f_bits(static_cast<const uint16_t*>(data)[i]) : static_cast<const float*>(data)[i];
    };
    // a weight that changes invalidates what holds its old device pointer:
    // the cached decision-tail pointers and every captured forward graph
    // (a plan's graph records the arena generation and is re-captured)
    tail_cache_ready = false;
    ++arena_gen;
    // work already queued on the engine's streams (a plan run) may still
    // read the buffer this upload replaces
    ck(cudaStreamSynchronize(stream), "sync");
    if (side) ck(cudaStreamSynchronize(side), "sync");
    Weight& wt = w[name];
    switch (role.kind) {
      case Kind::Linear:
      case Kind::Embed:
      case Kind::ActW1: {
        std::vector<uint16_t> h;
        const bool wi = name.find(".mlp.Wi.weight") != std::string::npos;
        if (wi) {
          // Gate/up co-tiling for the fused GeGLU epilogue: output tile j
          // (256 rows) holds gate rows 128j..128j+127 then the matching up
          // rows 2624+128j..; rows past 2624 in a half are zero.
          h.assign((size_t)2 * INTER_PAD * H, 0);
          for (int j = 0; j < INTER_PAD / 128; ++j)
            for (int r = 0; r < 128; ++r) {
              const int g = 128 * j + r;
              if (g >= INTER) continue;
              for (int c = 0; c < H; ++c) {
                h[((size_t)256 * j + r) * H + c] = f2h_or_copy(data, is_f16, (size_t)g * H + c);
                h[((size_t)256 * j + 128 + r) * H + c] = f2h_or_copy(data, is_f16, (size_t)(INTER + g) * H + c);
              }
            }
        } else {
          h.resize(el);
          for (size_t i = 0; i < el; ++i) h[i] = f2h_or_copy(data, is_f16, i);
        }
        wt.buf.alloc(h.size() * 2, "weight alloc");
        upload_sync(wt.buf.p, h.data(), h.size() * 2, "weight upload");
        if (role.kind == Kind::Linear) {
          const uint64_t rows = wi ? (uint64_t)2 * INTER_PAD : (uint64_t)role.shape[0];
          const uint64_t kdim = (uint64_t)role.shape[1];
          if (make_tmap_f16(&wt.tmap, wt.buf.p, rows, kdim, kGemmBBoxRows) != 0)
            throw Error(LAYA_E_CUDA, "tensor map encode failed for " + name);
          if (make_tmap_f16(&wt.tmap_narrow, wt.buf.p, rows, kdim, kGemmBBoxRowsNarrow) != 0)
            throw Error(LAYA_E_CUDA, "tensor map encode failed for " + name);
        }
        break;
      }
      case Kind::F32Vec:
      case Kind::F32Mat:
      case Kind::Rope: {
        std::vector<float> f(el);
        for (size_t i = 0; i < el; ++i) f[i] = f32_at(i);
        wt.buf.alloc(el * 4, "weight alloc");
        upload_sync(wt.buf.p, f.data(), el * 4, "weight upload");
        if (role.kind == Kind::Rope || name == "scorer.3.bias") wt.host = f;
        break;
      }
    }
    wt.present = true;
  }

  // A tensor as Tensors::f32 returns it (weights.rs:278-295): graph layout,
  // i.e. the 120 matmul weights of the transpose set (arch.rs:306-322)
  // transposed to [in, out] with dims as Tensors::dims reports them
  // (weights.rs:270-276); every other tensor as stored.  Transposed back to
  // the stored [out, in] layout, then uploaded like any stored tensor.
  void upload_graph(const std::string& name, const float* data, const int64_t* dims, int nd) {
    auto it = roles().find(name);
    if (it == roles().end()) throw Error(LAYA_E_LOAD, "unknown tensor name " + name);
    const std::vector<int64_t>& st = it->second.shape;
    if (!in_transpose_set(name) || st.size() != 2) {
      upload(name, data, false, dims, nd);
      return;
    }
    if (nd != 2 || dims[0] != st[1] || dims[1] != st[0])
      throw Error(LAYA_E_LOAD, fmt("tensor %s: graph-layout dims must be [%lld, %lld]", name.c_str(), (long long)st[1],
                                   (long long)st[0]));
    const size_t a = (size_t)st[0], c = (size_t)st[1];
    std::vector<float> v(a * c);
    // graph element (j, i) at j * a + i is stored element (i, j) at i * c + j
    for (size_t i = 0; i < a; ++i)
      for (size_t j = 0; j < c; ++j) v[i * c + j] = data[j * a + i];
    upload(name, v.data(), false, st.data(), 2);
  }

  static uint16_t f2h_or_copy(const void* data, bool is_f16, size_t i) {
    return is_f16 ? static_cast<const uint16_t*>(data)[i] : f2h_bits(static_cast<const float*>(data)[i]);
  }

  void finalize() {
    for (const auto& kv : roles()) {
      auto it = w.find(kv.first);
      if (it == w.end() || !it->second.present) throw Error(LAYA_E_LOAD, "no tensor named " + kv.first);
    }
    finalized = true;
    ensure_rope(512);
  }

  // graph.rs:62-84: cos/sin(p * freq[j]) in f32 with libm cosf/sinf.
  // Host -> device copy on the engine's stream, complete on return.  The
  // engine's streams are non-blocking: a cudaMemcpy or cudaMemset on the
  // legacy default stream is not ordered before their kernels (and from
  // pageable memory may return before its DMA lands), so every write into the
  // engine's buffers goes through its own stream.
  void upload_sync(void* dst, const void* src, size_t bytes, const char* what) {
    ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), what);
    ck(cudaStreamSynchronize(stream), what);
  }

  void ensure_rope(int len) {
    if (len <= rope_len) return;
    int n = rope_len ? rope_len : 512;
    while (n < len) n *= 2;
    const auto& ff = W("rope.freq_full").host;
    const auto& fs = W("rope.freq_sliding").host;
    std::vector<float> cf(n * 32), sf(n * 32), cs(n * 32), ss(n * 32);
    for (int p = 0; p < n; ++p)
      for (int j = 0; j < 32; ++j) {
        const float a = (float)p * ff[j];
        const float b = (float)p * fs[j];
        cf[p * 32 + j] = cosf(a);
        sf[p * 32 + j] = sinf(a);
        cs[p * 32 + j] = cosf(b);
        ss[p * 32 + j] = sinf(b);
      }
    ck(cudaStreamSynchronize(stream), "sync");
    // the tables move: graphs captured over the old ones must not replay
    ++arena_gen;
    for (auto* pr : {&cos_full, &sin_full, &cos_slide, &sin_slide}) pr->alloc((size_t)n * 32 * 4, "rope alloc");
    upload_sync(cos_full.p, cf.data(), cf.size() * 4, "rope upload");
    upload_sync(sin_full.p, sf.data(), sf.size() * 4, "rope upload");
    upload_sync(cos_slide.p, cs.data(), cs.size() * 4, "rope upload");
    upload_sync(sin_slide.p, ss.data(), ss.size() * 4, "rope upload");
    rope_len = n;
  }

  // ---- arena ----------------------------------------------------------------------
  void ensure_arena(const HostPlan& p) {
    ensure_rope(p.l);
    ensure_parts();
    const int rows = (p.R + kGemmBM - 1) / kGemmBM * kGemmBM;
    const int mk = (p.n * p.k + kGemmBM - 1) / kGemmBM * kGemmBM;
    if (rows <= cap_rows && mk <= cap_mk && p.n <= cap_n) return;
    ck(cudaStreamSynchronize(stream), "sync");
    cap_rows = std::max(rows, cap_rows);
    cap_mk = std::max(mk, cap_mk);
    cap_n = std::max(p.n, cap_n);
    ++arena_gen;
    const size_t R = cap_rows;
    x.alloc(R * H * 4, "arena x");
    t16.alloc(R * H * 2, "arena t16");
    qkv.alloc(R * 3 * H * 2, "arena qkv");
    ctx.alloc(R * H * 2, "arena ctx");
    gate.alloc(R * INTER * 2, "arena gate");
    hmlp.alloc(R * HEAD_INTER * 2, "arena hmlp");
    mk16.alloc((size_t)cap_mk * H * 2, "arena markers");
    partial.alloc((size_t)kScorerPartials * cap_mk * 4, "arena partial");
    out_logits.alloc((size_t)cap_mk * 4, "arena logits");
    out_act.alloc((size_t)cap_n * 2 * 4, "arena act");
    // on the engine's stream, so the clears precede the forward's kernels
    for (DevBuf* b : {&x, &t16, &qkv, &ctx, &gate, &hmlp, &mk16, &partial})
      ck(cudaMemsetAsync(b->p, 0, b->bytes, stream), "arena clear");
  }

  // The split-K part regions: allocated once, with a plan (never while a
  // stream is being captured).
  void ensure_parts() {
    if (parts_ready || !splitk_enabled()) return;
    for (int g = 0; g < 2; ++g) {
      parts[g].alloc((size_t)kPartRows * H * 4, "split-K parts");
      if (make_tmap_2d(&parts_map[g], parts[g].p, true, kPartRows, H, 32, kGemmOutBoxRows))
        throw Error(LAYA_E_CUDA, "tensor map encode failed for the split-K parts");
    }
    parts_ready = true;
  }

  // The split tail of a large residual GEMM of M rows: when its 256 x 256
  // tiles fill more than one wave of clusters but leave the last one at most
  // half full, the last tail_rb row blocks (covering those tiles) are cut
  // into `splits` K parts (2..4, at least 4 k-blocks each, within the part
  // region); splits < 2 means no tail split.
  void choose_tail(int M, int K, int& tail_rb, int& splits) const {
    tail_rb = 0;
    splits = 1;
    if (!parts_ready || !tailsplit_enabled()) return;
    const int num_m = (M + kGemmBM - 1) / kGemmBM, num_n = H / kGemmBN, tiles = num_m * num_n;
    const int clusters = num_sms / 2;
    const int rem = tiles % clusters;
    if (tiles <= clusters || rem == 0 || rem * 2 > clusters) return;
    tail_rb = (rem + num_n - 1) / num_n;
    int S = std::min(std::min(4, clusters / (tail_rb * num_n)), (K / kGemmBK) / 4);
    while (S > 1 && S * tail_rb * kGemmBM > kPartRows) --S;
    splits = S;
  }

  // K parts for a residual GEMM of M rows: 1 (no split) unless its tiles
  // fill at most half the clusters; then as many as fill the clusters, at
  // least 4 k-blocks each, at most splitk_max(), within the part region.
  int choose_splits(int M, int K) const {
    if (!parts_ready) return 1;
    const int num_m = (M + kGemmBM - 1) / kGemmBM, tiles = num_m * (H / kGemmBN);
    const int clusters = num_sms / 2;
    if (tiles == 0 || tiles * 2 > clusters) return 1;
    int S = std::min(std::min(clusters / tiles, (K / kGemmBK) / 4), splitk_max());
    while (S > 1 && S * num_m * kGemmBM > kPartRows) --S;
    return S;
  }

  void ensure_maps(DevicePlan& dp) {
    PlanMaps& m = dp.maps;
    if (m.gen == arena_gen) return;
    const HostPlan& p = dp.host;
    const uint64_t R = (uint64_t)p.R, nk = (uint64_t)p.n * p.k;
    const uint32_t ab = kGemmABoxRows, ob = kGemmOutBoxRows;
    bool bad = make_tmap_f16(&m.a_mk, mk16.p, nk, H, ab) != 0 ||
               make_tmap_2d(&m.qkv_rows, qkv.p, false, R, 3 * H, 64, kAttnTcBoxRows) != 0;
    for (size_t g = 0; g < p.groups.size() && !bad; ++g) {
      // each group's maps start at its first row and end at its last, so its
      // TMA stores never reach the other group's rows
      GroupMaps& q = m.g[g];
      const size_t r0 = (size_t)p.groups[g].row0;
      const uint64_t rows = (uint64_t)p.groups[g].rows;
      bad = make_tmap_f16(&q.a_t16, t16.as<__half>() + r0 * H, rows, H, ab) ||
            make_tmap_f16(&q.a_ctx, ctx.as<__half>() + r0 * H, rows, H, ab) ||
            make_tmap_f16(&q.a_gate, gate.as<__half>() + r0 * INTER, rows, INTER, ab) ||
            make_tmap_f16(&q.a_hmlp, hmlp.as<__half>() + r0 * HEAD_INTER, rows, HEAD_INTER, ab) ||
            make_tmap_2d(&q.o_qkv, qkv.as<__half>() + r0 * 3 * H, false, rows, 3 * H, 64, ob) ||
            make_tmap_2d(&q.o_x, x.as<float>() + r0 * H, true, rows, H, 32, ob) ||
            make_tmap_2d(&q.o_gate, gate.as<__half>() + r0 * INTER, false, rows, INTER, 64, ob) ||
            make_tmap_2d(&q.o_hmlp, hmlp.as<__half>() + r0 * HEAD_INTER, false, rows, HEAD_INTER, 64, ob);
    }
    if (bad) throw Error(LAYA_E_CUDA, "tensor map encode failed for the arena");
    m.gen = arena_gen;
  }

  // ---- the forward ---------------------------------------------------------------
  void gemm(int epi, const CUtensorMap& A, const Weight& Wt, const CUtensorMap& Out, int M, int N, int K, GemmArgs a,
            cudaStream_t s, int64_t& nl, int kind, const CUtensorMap* out2 = nullptr) {
    a.M = M;
    a.N = N;
    a.K = K;
    a.err = err.as<int>();
    if (stuck_next && stuck_kind == 0) {
      // the timeout test (see stuck_next)
      a.stuck = 1;
      a.wait_limit_ns = stuck_limit_ns;
      stuck_next = false;
    }
    // 256 x 128 tiles for the f16-output GEMMs of small batches, whose
    // 256 x 256 tiles would fill at most half the clusters: twice the
    // clusters stream the weights.  Large batches keep 256 x 256 (256 x 128
    // measured slower there: the smaller stages leave the TMA latency
    // exposed); the residual GEMMs of small batches split K instead.
    const int tiles256 = ((M + kGemmBM - 1) / kGemmBM) * (N / kGemmBN);
    const bool narrow = narrow_enabled() && tiles256 * 2 <= num_sms / 2 &&
                        (epi == kEpiQkvRope || epi == kEpiQkvBias || epi == kEpiGeglu || epi == kEpiBiasRelu);
    ck(launch_gemm(epi, GemmMaps{&A, narrow ? &Wt.tmap_narrow : &Wt.tmap, &Out, out2}, a, num_sms, s,
                   narrow ? kGemmBNNarrow : kGemmBN),
       "gemm launch");
    ++nl;
    mark(kind);
  }

  // Attention over the group's sequences: one launch for the tiles of
  // sequences of at most 128 tokens (single pass) and one of the flash
  // kernel for longer ones.
  void attention(const DevicePlan& dp, int gi, int window, cudaStream_t s, int64_t& nl) {
    const RowGroup& g = dp.host.groups[gi];
    const PlanLayout& L = dp.lay;
    const bool stuck = stuck_next && stuck_kind == 1;
    if (g.ntiles > 0) {
      AttnShortArgs sa{};
      sa.out = ctx.as<__half>();
      sa.tiles = dp.at<int2>(L.tiles) + g.tile0;
      sa.rowseq = dp.at<int>(L.rowseq);
      sa.seq_start = dp.at<int>(L.seq_start);
      sa.seq_len = dp.at<int>(L.seq_len);
      sa.num_tiles = g.ntiles;
      sa.window = window;
      sa.err = err.as<int>();
      if (stuck) {
        // the timeout test: this launch's loads first wait on a barrier
        // nothing completes, for stuck_limit_ns, then the kernel unwinds
        sa.stuck = 1;
        sa.wait_limit_ns = stuck_limit_ns;
      }
      ck(launch_attention_short(&dp.maps.qkv_rows, sa, num_sms, s), "attention");
      ++nl;
      mark(kProfAttn);
    }
    if (g.nitems > 0) {
      AttnArgs aa{};
      aa.out = ctx.as<__half>();
      aa.items = dp.at<int4>(L.items) + g.item0;
      aa.num_items = g.nitems;
      aa.window = window;
      aa.err = err.as<int>();
      if (stuck) {
        aa.stuck = 1;
        aa.wait_limit_ns = stuck_limit_ns;
      }
      ck(launch_attention_tc(&dp.maps.qkv_rows, aa, num_sms, s), "attention");
      ++nl;
      mark(kProfAttn);
    }
    if (stuck) stuck_next = false;
  }

  // LayerNorm of row group gi's residual rows into `out`; first adds the
  // split-K parts the group's last residual GEMM left, if any.
  void row_ln(int gi, float* xin, const std::string& wname, const float* b, __half* out, int rows, cudaStream_t s,
              int64_t& nl) {
    if (pend[gi].nparts > 0) {
      ck(launch_ln_parts(xin, pend[gi], W(wname).buf.as<float>(), b, EPS, out, rows, s), "ln parts");
      pend[gi] = PendingParts();
    } else {
      ck(launch_ln(xin, nullptr, W(wname).buf.as<float>(), b, EPS, out, rows, s), "ln");
    }
    ++nl;
    mark(kProfNorm);
  }

  // x += A . W^T for an encoder residual GEMM (no bias).  With `defer`
  // (a LayerNorm of the same rows comes next) and a small M, the K loop is
  // split and the sums stay pending for that LayerNorm.
  void resid_gemm(int gi, const CUtensorMap& A, const Weight& Wt, const CUtensorMap& Out, int R, int K, cudaStream_t s,
                  int64_t& nl, int kind, bool defer, const float* bias = nullptr) {
    GemmArgs r{};
    r.ldo = H;
    r.bias = bias;
    const int S = defer ? choose_splits(R, K) : 1;
    if (S < 2) {
      int tail_rb = 0, ts = 0;
      if (defer) choose_tail(R, K, tail_rb, ts);
      if (ts < 2) {
        gemm(kEpiResid, A, Wt, Out, R, H, K, r, s, nl, kind);
        return;
      }
      if (pend[gi].nparts > 0) throw Error(LAYA_E_STATE, "split-K parts of an earlier GEMM were not consumed");
      const int num_m = (R + kGemmBM - 1) / kGemmBM, num_n = H / kGemmBN;
      r.splits = ts;
      r.main_tiles = (num_m - tail_rb) * num_n;
      r.tail_row0 = (num_m - tail_rb) * kGemmBM;
      r.split_rows = tail_rb * kGemmBM;
      gemm(kEpiResidTail, A, Wt, Out, R, H, K, r, s, nl, kind, &parts_map[gi]);
      pend[gi] = PendingParts{parts[gi].as<float>(), ts, (size_t)r.split_rows * H, r.tail_row0};
      return;
    }
    if (pend[gi].nparts > 0) throw Error(LAYA_E_STATE, "split-K parts of an earlier GEMM were not consumed");
    r.splits = S;
    r.split_rows = (R + kGemmBM - 1) / kGemmBM * kGemmBM;
    gemm(kEpiPartial, A, Wt, parts_map[gi], R, H, K, r, s, nl, kind);
    pend[gi] = PendingParts{parts[gi].as<float>(), S, (size_t)r.split_rows * H};
  }

  // Encoder layer `layer` (graph.rs:104-123) for row group gi on stream s.
  // In the forward (`embedded`), layer 0's input norm is the embedding norm,
  // already applied by embed_ln.
  // Wo_mlp's split-K parts, if any, stay pending for the LayerNorm after
  // this layer (the next layer's input norm, or the final norm); a caller
  // that reads the residual stream first folds them in (fold_parts).
  void enc_layer(const DevicePlan& dp, int gi, int layer, cudaStream_t s, int64_t& nl, bool embedded = true) {
    const RowGroup& g = dp.host.groups[gi];
    const GroupMaps& M = dp.maps.g[gi];
    const size_t r0 = (size_t)g.row0;
    const int R = g.rows;
    const bool global = layer % GLOBAL_EVERY == 0;
    float* xg = x.as<float>() + r0 * H;
    __half* tg = t16.as<__half>() + r0 * H;
    if (layer > 0) {
      row_ln(gi, xg, attn_norm(layer), nullptr, tg, R, s, nl);
    } else if (!embedded) {
      // layer 0 alone: its input norm is the embedding norm, and its residual
      // base is the normed input (graph.rs:112-113), so x itself is normed
      ck(launch_ln_inplace(xg, W(attn_norm(0)).buf.as<float>(), EPS, tg, R, s), "ln");
      ++nl;
      mark(kProfNorm);
    }
    GemmArgs q{};
    q.ldo = 3 * H;
    q.pos = dp.at<int>(dp.lay.pos) + r0;
    q.cosb = global ? cos_full.as<float>() : cos_slide.as<float>();
    q.sinb = global ? sin_full.as<float>() : sin_slide.as<float>();
    q.scale = SCALE;
    gemm(kEpiQkvRope, M.a_t16, W(fmt("encoder.layers.%d.attn.Wqkv.weight", layer)), M.o_qkv, R, 3 * H, H, q, s, nl,
         kProfQkv);
    attention(dp, gi, global ? -1 : WINDOW, s, nl);
    resid_gemm(gi, M.a_ctx, W(fmt("encoder.layers.%d.attn.Wo.weight", layer)), M.o_x, R, H, s, nl, kProfWo, true);
    row_ln(gi, xg, fmt("encoder.layers.%d.mlp_norm.weight", layer), nullptr, tg, R, s, nl);
    GemmArgs gg{};
    gg.ldo = INTER;
    gg.n_valid = INTER;
    gemm(kEpiGeglu, M.a_t16, W(fmt("encoder.layers.%d.mlp.Wi.weight", layer)), M.o_gate, R, 2 * INTER_PAD, H, gg, s,
         nl, kProfWi);
    resid_gemm(gi, M.a_gate, W(fmt("encoder.layers.%d.mlp.Wo.weight", layer)), M.o_x, R, INTER, s, nl, kProfWo2,
               true);
  }

  // Adds row group gi's pending split-K parts to its residual rows.
  void fold_parts(const DevicePlan& dp, int gi, cudaStream_t s, int64_t& nl) {
    if (pend[gi].nparts == 0) return;
    const RowGroup& g = dp.host.groups[gi];
    ck(launch_add_parts(x.as<float>() + (size_t)g.row0 * H, pend[gi], g.rows, s), "add parts");
    pend[gi] = PendingParts();
    ++nl;
    mark(kProfNorm);
  }

  static std::string hn(int i, const char* s) { return fmt("head.layers.%d.%s", i, s); }

  // Final norm + type embedding (graph.rs:126-128) fused with head layer 0's
  // norm1, for row group gi.
  void final_norm(const DevicePlan& dp, int gi, cudaStream_t s, int64_t& nl) {
    const RowGroup& g = dp.host.groups[gi];
    const size_t r0 = (size_t)g.row0;
    ck(launch_final_ln(x.as<float>() + r0 * H, W("encoder.final_norm.weight").buf.as<float>(),
                       W("type_emb.weight").buf.as<__half>(), dp.at<uint8_t>(dp.lay.rowtype) + r0,
                       W(hn(0, "norm1.weight")).buf.as<float>(), W(hn(0, "norm1.bias")).buf.as<float>(), EPS,
                       t16.as<__half>() + r0 * H, g.rows, s, pend[gi]),
       "final_ln");
    pend[gi] = PendingParts();
    ++nl;
    mark(kProfNorm);
  }

  // Head layer hl (graph.rs:131-152: a pre-norm transformer layer with
  // biases, global attention and a ReLU MLP) for row group gi.
  void head_layer(const DevicePlan& dp, int gi, int hl, cudaStream_t s, int64_t& nl) {
    const RowGroup& g = dp.host.groups[gi];
    const GroupMaps& M = dp.maps.g[gi];
    const size_t r0 = (size_t)g.row0;
    const int R = g.rows;
    float* xg = x.as<float>() + r0 * H;
    __half* tg = t16.as<__half>() + r0 * H;
    if (hl > 0) row_ln(gi, xg, hn(hl, "norm1.weight"), W(hn(hl, "norm1.bias")).buf.as<float>(), tg, R, s, nl);
    GemmArgs q{};
    q.ldo = 3 * H;
    q.bias = W(hn(hl, "self_attn.in_proj_bias")).buf.as<float>();
    q.scale = SCALE;
    gemm(kEpiQkvBias, M.a_t16, W(hn(hl, "self_attn.in_proj_weight")), M.o_qkv, R, 3 * H, H, q, s, nl, kProfHead);
    attention(dp, gi, -1, s, nl);
    resid_gemm(gi, M.a_ctx, W(hn(hl, "self_attn.out_proj.weight")), M.o_x, R, H, s, nl, kProfHead, true,
               W(hn(hl, "self_attn.out_proj.bias")).buf.as<float>());
    row_ln(gi, xg, hn(hl, "norm2.weight"), W(hn(hl, "norm2.bias")).buf.as<float>(), tg, R, s, nl);
    GemmArgs f{};
    f.ldo = HEAD_INTER;
    f.bias = W(hn(hl, "linear1.bias")).buf.as<float>();
    gemm(kEpiBiasRelu, M.a_t16, W(hn(hl, "linear1.weight")), M.o_hmlp, R, HEAD_INTER, H, f, s, nl, kProfHead);
    // its split-K parts (small batches) stay pending for the next head
    // layer's norm1; after the last head layer they are folded in before the
    // scorer's gathered LayerNorm
    resid_gemm(gi, M.a_hmlp, W(hn(hl, "linear2.weight")), M.o_x, R, HEAD_INTER, s, nl, kProfHead, true,
               W(hn(hl, "linear2.bias")).buf.as<float>());
  }

  // Scorer over the gathered marker rows and the act head (graph.rs:154-186),
  // for the whole batch.
  void scorer_tail(const DevicePlan& dp, cudaStream_t s, int64_t& nl) {
    const HostPlan& p = dp.host;
    const PlanLayout& L = dp.lay;
    const int nk = p.n * p.k;
    ck(launch_ln(x.as<float>(), dp.at<int>(L.mk_row), W("scorer.0.weight").buf.as<float>(),
                 W("scorer.0.bias").buf.as<float>(), EPS, mk16.as<__half>(), nk, s),
       "scorer ln");
    ++nl;
    mark(kProfNorm);
    GemmArgs sa{};
    sa.out = partial.p;
    sa.ldo = cap_mk;
    sa.bias = W("scorer.1.bias").buf.as<float>();
    sa.wvec = W("scorer.3.weight").buf.as<float>();
    gemm(kEpiScorer, dp.maps.a_mk, W("scorer.1.weight"), dp.maps.a_mk, nk, H, H, sa, s, nl, kProfHead);
    TailArgs t{};
    t.partial = partial.as<float>();
    t.ldp = cap_mk;
    t.score_bias = W("scorer.3.bias").host[0];
    t.mmask = dp.at<int8_t>(L.mmask);
    t.cls_row = dp.at<int>(L.cls_row);
    t.x = x.as<float>();
    t.w1 = W("act_head.0.weight").buf.as<__half>();
    t.b1 = W("act_head.0.bias").buf.as<float>();
    t.w2 = W("act_head.2.weight").buf.as<float>();
    t.b2 = W("act_head.2.bias").buf.as<float>();
    t.logits = out_logits.as<float>();
    t.act = out_act.as<float>();
    t.n = p.n;
    t.k = p.k;
    ck(launch_tail(t, s), "tail");
    ++nl;
    mark(kProfTail);
  }

  // Streams of the row groups: group 0 on the engine stream, group 1 on the
  // side stream, forked from and joined back into the engine stream.  With
  // `concurrent` false (taps, per-launch profiling) both run on the engine
  // stream, interleaved layer by layer.
  cudaStream_t group_stream(int gi, bool concurrent) const { return concurrent && gi > 0 ? side : stream; }

  void fork(bool concurrent) {
    if (!concurrent) return;
    ck(cudaEventRecord(ev_fork, stream), "fork record");
    ck(cudaStreamWaitEvent(side, ev_fork, 0), "fork wait");
  }

  void join(bool concurrent) {
    if (!concurrent) return;
    ck(cudaEventRecord(ev_join, side), "join record");
    ck(cudaStreamWaitEvent(stream, ev_join, 0), "join wait");
  }

  // Enqueues one forward of plan `dp` (graph.rs:86-186).
  int64_t enqueue(DevicePlan& dp, laya_tap_fn tap = nullptr, void* user = nullptr) {
    ensure_maps(dp);
    const HostPlan& p = dp.host;
    const int G = (int)p.groups.size();
    const bool conc = G > 1 && !tap && !prof_ev;
    int64_t nl = 0;
    fork(conc);
    for (int gi = 0; gi < G; ++gi) {
      const RowGroup& g = p.groups[gi];
      const size_t r0 = (size_t)g.row0;
      ck(launch_embed_ln(W("encoder.embeddings.tok_embeddings.weight").buf.as<__half>(),
                         dp.at<int>(dp.lay.tok) + r0, W(attn_norm(0)).buf.as<float>(), EPS, x.as<float>() + r0 * H,
                         t16.as<__half>() + r0 * H, g.rows, group_stream(gi, conc)),
         "embed_ln");
      ++nl;
      mark(kProfNorm);
    }
    pend[0] = pend[1] = PendingParts();
    for (int layer = 0; layer < NLAYER; ++layer) {
      for (int gi = 0; gi < G; ++gi) enc_layer(dp, gi, layer, group_stream(gi, conc), nl);
      if (tap) {
        // taps read the residual stream after each layer
        for (int gi = 0; gi < G; ++gi) fold_parts(dp, gi, group_stream(gi, conc), nl);
        emit_rows(dp, fmt("enc.%d", layer).c_str(), tap, user);
      }
    }
    for (int gi = 0; gi < G; ++gi) final_norm(dp, gi, group_stream(gi, conc), nl);
    if (tap) emit_rows(dp, "final", tap, user);
    for (int hl = 0; hl < HEAD_LAYERS; ++hl) {
      for (int gi = 0; gi < G; ++gi) head_layer(dp, gi, hl, group_stream(gi, conc), nl);
      if (tap) {
        for (int gi = 0; gi < G; ++gi) fold_parts(dp, gi, group_stream(gi, conc), nl);
        emit_rows(dp, fmt("head.%d", hl).c_str(), tap, user);
      }
    }
    for (int gi = 0; gi < G; ++gi) fold_parts(dp, gi, group_stream(gi, conc), nl);
    join(conc);
    scorer_tail(dp, stream, nl);
    if (pend[0].nparts || pend[1].nparts) throw Error(LAYA_E_STATE, "split-K parts left pending after the forward");
    return nl;
  }

  // One encoder layer (0..27) on the arena's residual stream, the body of the
  // layer loop of graph.rs:103-123: LN, QKV + RoPE, attention, Wo + residual,
  // LN, Wi + GeGLU, Wo_mlp + residual.
  int64_t enqueue_layer(DevicePlan& dp, int layer) {
    ensure_maps(dp);
    const int G = (int)dp.host.groups.size();
    const bool conc = G > 1 && !prof_ev;
    int64_t nl = 0;
    fork(conc);
    pend[0] = pend[1] = PendingParts();
    for (int gi = 0; gi < G; ++gi) {
      enc_layer(dp, gi, layer, group_stream(gi, conc), nl, false);
      fold_parts(dp, gi, group_stream(gi, conc), nl);
    }
    join(conc);
    return nl;
  }

  // Diagnostic: copies the residual stream back and scatters it to padded rows.
  void emit_rows(const DevicePlan& dp, const char* stage, laya_tap_fn tap, void* user) {
    const HostPlan& p = dp.host;
    std::vector<float> c((size_t)p.R * H), o((size_t)p.n * p.l * H, 0.0f);
    ck(cudaMemcpyAsync(c.data(), x.p, c.size() * 4, cudaMemcpyDeviceToHost, stream), "tap copy");
    ck(cudaStreamSynchronize(stream), "tap sync");
    for (int b = 0; b < p.n; ++b)
      memcpy(&o[(size_t)b * p.l * H], &c[(size_t)p.seq_start[b] * H], (size_t)p.seq_len[b] * H * 4);
    tap(user, stage, o.data(), o.size());
  }

  // Packs the plan into pinned staging and copies it to device memory.  The
  // staging buffer is reused: every caller synchronizes the stream before
  // the next upload (plan_create here, forward in read_outputs).
  void upload_plan(DevicePlan& dp, bool use_engine_buffer) {
    dp.lay = layout_for(dp.host);
    if (staging_bytes < dp.lay.total) {
      ck(cudaStreamSynchronize(stream), "sync");
      if (staging) cudaFreeHost(staging);
      staging = nullptr;
      staging_bytes = 0;
      ck(cudaMallocHost(&staging, dp.lay.total * 2), "pinned staging");
      staging_bytes = dp.lay.total * 2;
    }
    pack(dp.host, dp.lay, staging);
    if (use_engine_buffer) {
      if (plan_buf.bytes < dp.lay.total) {
        ck(cudaStreamSynchronize(stream), "sync");
        plan_buf.alloc(dp.lay.total * 2, "plan buffer");
      }
      dp.base = plan_buf.as<uint8_t>();
    } else {
      dp.own.alloc(dp.lay.total, "plan buffer");
      dp.base = dp.own.as<uint8_t>();
    }
    ck(cudaMemcpyAsync(dp.base, staging, dp.lay.total, cudaMemcpyHostToDevice, stream), "plan upload");
    if (!use_engine_buffer) ck(cudaStreamSynchronize(stream), "plan upload sync");
  }

  // Runs the plan `steps` times with an event after every launch; sums the
  // device time between consecutive events per launch kind.
  void profile(DevicePlan& dp, int steps, double* ms, int64_t* launches) {
    for (int i = 0; i < 8; ++i) {
      ms[i] = 0;
      launches[i] = 0;
    }
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
    prof_ev = &ev;
    prof_kind = &kind;
    try {
      for (int s = 0; s < steps; ++s) {
        mark(-1);
        enqueue(dp);
      }
      prof_ev = nullptr;
      prof_kind = nullptr;
      ck(cudaStreamSynchronize(stream), "profile sync");
      for (size_t i = 1; i < ev.size(); ++i) {
        if (kind[i] < 0) continue;
        float t = 0;
        ck(cudaEventElapsedTime(&t, ev[i - 1], ev[i]), "event elapsed");
        ms[kind[i]] += t;
        launches[kind[i]] += 1;
      }
    } catch (...) {
      prof_ev = nullptr;
      prof_kind = nullptr;
      cudaStreamSynchronize(stream);
      for (auto e : ev) cudaEventDestroy(e);
      throw;
    }
    for (auto e : ev) cudaEventDestroy(e);
  }

  void check_device_error() {
    int e = 0;
    ck(cudaMemcpyAsync(&e, err.p, sizeof(int), cudaMemcpyDeviceToHost, stream), "error word read");
    ck(cudaStreamSynchronize(stream), "forward sync");
    if (e != 0) {
      ck(cudaMemsetAsync(err.p, 0, sizeof(int), stream), "error word reset");
      ck(cudaStreamSynchronize(stream), "sync");
      throw Error(LAYA_E_DEVICE_TIMEOUT, fmt("a device-side wait expired (code %d)", e));
    }
  }

  void read_outputs(const HostPlan& p, float* logits, float* act) {
    const size_t nl = (size_t)p.n * p.k, na = (size_t)p.n * 2;
    if (pinned_out_floats < nl + na) {
      if (pinned_out) cudaFreeHost(pinned_out);
      pinned_out = nullptr;
      ck(cudaMallocHost(&pinned_out, (nl + na) * 4), "pinned alloc");
      pinned_out_floats = nl + na;
    }
    ck(cudaMemcpyAsync(pinned_out, out_logits.p, nl * 4, cudaMemcpyDeviceToHost, stream), "logits copy");
    ck(cudaMemcpyAsync(pinned_out + nl, out_act.p, na * 4, cudaMemcpyDeviceToHost, stream), "act copy");
    check_device_error();
    memcpy(logits, pinned_out, nl * 4);
    memcpy(act, pinned_out + nl, na * 4);
  }

  // Everything the forward's launches take as arguments besides the plan
  // buffer's contents: the batch shape, row groups and attention work
  // counts (grids, tensor-map extents, split-K choices), the plan buffer's
  // layout and address, and the arena generation.
  std::vector<int64_t> forward_graph_key(const DevicePlan& dp) const {
    const HostPlan& p = dp.host;
    const PlanLayout& L = dp.lay;
    std::vector<int64_t> k = {p.n, p.k, p.R, p.ntiles, p.nitems, (int64_t)arena_gen,
                              (int64_t)(uintptr_t)dp.base, (int64_t)L.tok, (int64_t)L.pos, (int64_t)L.seq_start,
                              (int64_t)L.seq_len, (int64_t)L.cls_row, (int64_t)L.mk_row, (int64_t)L.tiles,
                              (int64_t)L.items, (int64_t)L.rowtype, (int64_t)L.mmask, (int64_t)L.rowseq,
                              (int64_t)L.total, (int64_t)rope_len, parts_ready ? 1 : 0};
    for (const RowGroup& g : p.groups) {
      k.push_back(g.row0);
      k.push_back(g.rows);
      k.push_back(g.tile0);
      k.push_back(g.ntiles);
      k.push_back(g.item0);
      k.push_back(g.nitems);
    }
    return k;
  }

  // The cached graph of this forward's shape, capturing it on the shape's
  // second call; nullptr: run it eagerly.
  cudaGraphExec_t forward_graph(DevicePlan& dp) {
    if (!forward_graphs_enabled()) return nullptr;
    fwd_graphs.erase(std::remove_if(fwd_graphs.begin(), fwd_graphs.end(),
                                    [&](FwdGraph& g) {
                                      if (g.gen == arena_gen) return false;
                                      if (g.exec) cudaGraphExecDestroy(g.exec);
                                      return true;
                                    }),
                     fwd_graphs.end());
    const std::vector<int64_t> key = forward_graph_key(dp);
    for (auto& g : fwd_graphs)
      if (g.key == key) {
        g.last_use = ++fwd_clock;
        return g.exec;
      }
    if (fwd_seen.size() > 4096) fwd_seen.clear();
    if (++fwd_seen[key] < 2) return nullptr;  // a shape seen once runs eagerly
    cudaGraph_t graph = nullptr;
    ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      enqueue(dp);
    } catch (...) {
      cudaStreamEndCapture(stream, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    ck(cudaStreamEndCapture(stream, &graph), "end capture");
    cudaGraphExec_t exec = nullptr;
    cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    ck(ie, "graph instantiate");
    if (fwd_graphs.size() >= kForwardGraphs) {
      auto lru = std::min_element(fwd_graphs.begin(), fwd_graphs.end(),
                                  [](const FwdGraph& a, const FwdGraph& b) { return a.last_use < b.last_use; });
      cudaGraphExecDestroy(lru->exec);
      fwd_graphs.erase(lru);
    }
    fwd_graphs.push_back(FwdGraph{key, exec, arena_gen, ++fwd_clock});
    return exec;
  }

  void forward(const laya_req* q, float* logits, float* act, laya_tap_fn tap, void* user) {
    if (!finalized) throw Error(LAYA_E_STATE, "engine has no weights (call laya_finalize)");
    if (!logits || !act) throw Error(LAYA_E_INVALID, "null output buffer");
    set_device();
    DevicePlan dp;
    dp.host = make_plan(q);
    ensure_arena(dp.host);
    upload_plan(dp, true);
    // taps read the stream between layers and the timeout test needs its
    // stuck launch: both run eagerly
    cudaGraphExec_t g = (tap || stuck_next) ? nullptr : forward_graph(dp);
    if (g)
      ck(cudaGraphLaunch(g, stream), "graph launch");
    else
      enqueue(dp, tap, user);
    read_outputs(dp.host, logits, act);
    if (tap) {
      tap(user, "logits", logits, (size_t)dp.host.n * dp.host.k);
      tap(user, "act", act, (size_t)dp.host.n * 2);
    }
  }
};

void load_gguf(Engine& e, const std::string& path) {
  GgufFile g(path);
  // ModelMeta::from_header (weights.rs:138-222)
  const GgufValue* arch = g.get("general.architecture");
  if (!arch || !arch->has_s || arch->s != "laya")
    throw Error(LAYA_E_LOAD, fmt("%s: general.architecture is %s, want \"laya\"", path.c_str(),
                                 arch && arch->has_s ? ("\"" + arch->s + "\"").c_str() : "\"\""));
  const std::pair<const char*, uint64_t> nums[] = {
      {"laya.hidden_size", H},         {"laya.num_layers", NLAYER},       {"laya.num_heads", NH},
      {"laya.head_dim", HD},           {"laya.intermediate_size", INTER}, {"laya.vocab_size", NVOCAB},
      {"laya.sliding_window", WINDOW}, {"laya.global_layer_every", GLOBAL_EVERY},
      {"laya.head_layers", HEAD_LAYERS}, {"laya.act_input_features", ACT_INPUT},
      {"laya.question_types", QTYPES}, {"laya.max_len", 512}, {"laya.head_max_len", 192},
      {"laya.max_prefixes", 6}};
  for (const auto& kv : nums) {
    const GgufValue* v = g.get(kv.first);
    if (!v) throw Error(LAYA_E_LOAD, fmt("%s: missing metadata %s", path.c_str(), kv.first));
    if (!v->has_u) throw Error(LAYA_E_LOAD, fmt("%s: metadata %s is not an integer", path.c_str(), kv.first));
    if (v->u != kv.second)
      throw Error(LAYA_E_LOAD, fmt("%s: metadata %s is %llu but this build pins %llu", path.c_str(), kv.first,
                                   (unsigned long long)v->u, (unsigned long long)kv.second));
  }
  const std::pair<const char*, float> flts[] = {{"laya.attention_scale", SCALE}, {"laya.layer_norm_epsilon", EPS}};
  for (const auto& kv : flts) {
    const GgufValue* v = g.get(kv.first);
    if (!v) throw Error(LAYA_E_LOAD, fmt("%s: missing metadata %s", path.c_str(), kv.first));
    if (!v->has_f) throw Error(LAYA_E_LOAD, fmt("%s: metadata %s is not a float", path.c_str(), kv.first));
    const float got = (float)v->f;
    uint32_t gb, wb;
    memcpy(&gb, &got, 4);
    memcpy(&wb, &kv.second, 4);
    if (gb != wb)
      throw Error(LAYA_E_LOAD, fmt("%s: metadata %s is %g but this build pins %g", path.c_str(), kv.first, got,
                                   kv.second));
  }
  for (int i = 0; i < 3; ++i) {
    const GgufValue* v = g.get(fmt("laya.temperature.%d", i));
    if (!v || !v->has_f) throw Error(LAYA_E_LOAD, fmt("%s: missing metadata laya.temperature.%d", path.c_str(), i));
    e.temperature[i] = (float)v->f;
  }
  if (const GgufValue* v = g.get("laya.temperature_by_options"); v && v->has_s) e.temperature_by_options = v->s;
  if (const GgufValue* v = g.get("general.file_type"); v && v->has_u) e.file_type = (int)v->u;
  if (e.file_type != 0 && e.file_type != 1)
    throw Error(LAYA_E_LOAD, fmt("general.file_type is %d, but this build only handles 0 (F32) and 1 (mostly F16)",
                                 e.file_type));
  std::vector<uint8_t> bytes;
  for (const auto& kv : roles()) {
    const GgufTensor* t = g.tensor(kv.first);
    if (!t) throw Error(LAYA_E_LOAD, path + ": no tensor named " + kv.first);
    if (t->ty != 0 && t->ty != 1 && t->ty != 30)
      throw Error(LAYA_E_LOAD, fmt("%s: tensor %s has type %u, which this build does not decode", path.c_str(),
                                   kv.first.c_str(), t->ty));
    bytes.resize(t->nbytes());
    g.read_bytes(*t, bytes.data());
    auto sd = t->stored_dims();
    if (t->ty == 30) {  // bf16 -> f32 (gguf.rs:560-563)
      std::vector<float> f(t->elems());
      const uint16_t* b = reinterpret_cast<const uint16_t*>(bytes.data());
      for (size_t i = 0; i < f.size(); ++i) {
        uint32_t u = (uint32_t)b[i] << 16;
        memcpy(&f[i], &u, 4);
      }
      e.upload(kv.first, f.data(), false, sd.data(), (int)sd.size());
    } else {
      e.upload(kv.first, bytes.data(), t->ty == 1, sd.data(), (int)sd.size());
    }
  }
  e.finalize();
}

Engine* open_engine(int device) {
  int n = 0;
  ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) throw Error(LAYA_E_INVALID, fmt("device %d out of range (%d devices)", device, n));
  std::unique_ptr<Engine> e(new Engine());
  e->device = device;
  e->set_device();
  cudaDeviceProp prop;
  ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    throw Error(LAYA_E_CUDA, fmt("device %d is sm_%d%d; this build targets sm_100a (B200)", device, prop.major,
                                 prop.minor));
  e->device_name = prop.name;
  e->num_sms = prop.multiProcessorCount;
  ck(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream create");
  ck(cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking), "stream create");
  ck(cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming), "event create");
  ck(cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming), "event create");
  e->err.alloc(256, "error word");
  ck(cudaMemsetAsync(e->err.p, 0, 256, e->stream), "error word clear");
  ck(cudaStreamSynchronize(e->stream), "sync");
  return e.release();
}

}  // namespace laya

using laya::Engine;
using laya::Error;
using laya::guard;

struct laya_engine {
  Engine* e;
};
struct laya_plan {
  laya::DevicePlan dp;
};

namespace laya {
// Fills *out with the engine's decision-tail weights; returns false (with the
// reason in laya_last_error) when the engine has no weights yet.
bool engine_tail_weights(laya_engine* e, TailWeights* out, int* status) {
  *status = guard([&] {
    if (!e) throw Error(LAYA_E_INVALID, "null engine");
    if (!e->e->finalized) throw Error(LAYA_E_STATE, "engine has no weights (call laya_finalize)");
    *out = e->e->tail_weights();
  });
  return *status == LAYA_OK;
}

void set_last_error(const char* msg) { g_err = msg; }
}  // namespace laya

extern "C" {

const char* laya_last_error(void) { return laya::g_err.c_str(); }

int laya_open(int device, const char* gguf_path, laya_engine** out) {
  return guard([&] {
    if (!out || !gguf_path) throw Error(LAYA_E_INVALID, "null argument");
    *out = nullptr;
    std::unique_ptr<Engine> e(laya::open_engine(device));
    laya::load_gguf(*e, gguf_path);
    *out = new laya_engine{e.release()};
  });
}

int laya_open_empty(int device, laya_engine** out) {
  return guard([&] {
    if (!out) throw Error(LAYA_E_INVALID, "null argument");
    *out = new laya_engine{laya::open_engine(device)};
  });
}

int laya_upload_weight_f16(laya_engine* e, const char* name, const uint16_t* data, const int64_t* dims, int nd) {
  return guard([&] {
    if (!e || !name || !data || !dims || nd <= 0 || nd > 4) throw Error(LAYA_E_INVALID, "bad argument");
    e->e->set_device();
    e->e->upload(name, data, true, dims, nd);
  });
}

int laya_upload_weight_f32(laya_engine* e, const char* name, const float* data, const int64_t* dims, int nd) {
  return guard([&] {
    if (!e || !name || !data || !dims || nd <= 0 || nd > 4) throw Error(LAYA_E_INVALID, "bad argument");
    e->e->set_device();
    e->e->upload(name, data, false, dims, nd);
  });
}

int laya_upload_weight_f32_graph(laya_engine* e, const char* name, const float* data, const int64_t* dims,
                                 int nd) {
  return guard([&] {
    if (!e || !name || !data || !dims || nd <= 0 || nd > 4) throw Error(LAYA_E_INVALID, "bad argument");
    e->e->set_device();
    e->e->upload_graph(name, data, dims, nd);
  });
}

int laya_finalize(laya_engine* e) {
  return guard([&] {
    if (!e) throw Error(LAYA_E_INVALID, "null engine");
    e->e->set_device();
    e->e->finalize();
  });
}

int laya_forward(laya_engine* e, const laya_req* req, float* logits, float* act) {
  return guard([&] {
    if (!e) throw Error(LAYA_E_INVALID, "null engine");
    e->e->forward(req, logits, act, nullptr, nullptr);
  });
}

int laya_forward_tapped(laya_engine* e, const laya_req* req, float* logits, float* act, laya_tap_fn fn,
                        void* user) {
  return guard([&] {
    if (!e || !fn) throw Error(LAYA_E_INVALID, "null argument");
    e->e->forward(req, logits, act, fn, user);
  });
}

int laya_info(laya_engine* e, char* buf, size_t len) {
  return guard([&] {
    if (!e || !buf || len == 0) throw Error(LAYA_E_INVALID, "null argument");
    const Engine& g = *e->e;
    std::string s = laya::fmt(
        "{\"id\":\"cuda\",\"device\":\"%s (cuda:%d, %d SMs)\",\"dtype\":\"%s\",\"layers\":%d,"
        "\"calibration\":{\"temperature\":[%.9g,%.9g,%.9g],\"by_options\":%s}}",
        g.device_name.c_str(), g.device, g.num_sms, g.file_type == 0 ? "fp32" : "fp16", laya::NLAYER,
        g.temperature[0], g.temperature[1], g.temperature[2], g.temperature_by_options.c_str());
    if (s.size() + 1 > len) throw Error(LAYA_E_INVALID, "info buffer too small");
    memcpy(buf, s.c_str(), s.size() + 1);
  });
}

void laya_close(laya_engine* e) {
  if (!e) return;
  if (e->e) {
    cudaSetDevice(e->e->device);
    delete e->e;
  }
  delete e;
}

int laya_plan_create(laya_engine* e, const laya_req* req, laya_plan** out) {
  return guard([&] {
    if (!e || !out) throw Error(LAYA_E_INVALID, "null argument");
    Engine& g = *e->e;
    if (!g.finalized) throw Error(LAYA_E_STATE, "engine has no weights (call laya_finalize)");
    g.set_device();
    std::unique_ptr<laya_plan> p(new laya_plan());
    p->dp.host = laya::make_plan(req);
    g.ensure_arena(p->dp.host);
    g.upload_plan(p->dp, false);
    *out = p.release();
  });
}

int laya_plan_run(laya_engine* e, laya_plan* p) {
  return guard([&] {
    if (!e || !p) throw Error(LAYA_E_INVALID, "null argument");
    Engine& g = *e->e;
    g.set_device();
    g.ensure_arena(p->dp.host);
    if (p->dp.graph && p->dp.graph_arena_gen != g.arena_gen) {
      // the arena moved since capture: the graph holds stale pointers
      cudaGraphExecDestroy(p->dp.graph);
      p->dp.graph = nullptr;
    }
    if (p->dp.graph) {
      laya::ck(cudaGraphLaunch(p->dp.graph, g.stream), "graph launch");
    } else {
      p->dp.launches = g.enqueue(p->dp);
    }
  });
}

int laya_plan_capture(laya_engine* e, laya_plan* p) {
  return guard([&] {
    if (!e || !p) throw Error(LAYA_E_INVALID, "null argument");
    Engine& g = *e->e;
    g.set_device();
    g.ensure_arena(p->dp.host);
    // one eager run first: per-device kernel attributes are set outside capture
    g.enqueue(p->dp);
    laya::ck(cudaStreamSynchronize(g.stream), "sync");
    g.check_device_error();
    cudaGraph_t graph = nullptr;
    laya::ck(cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    int64_t nl = 0;
    try {
      nl = g.enqueue(p->dp);
    } catch (...) {
      cudaStreamEndCapture(g.stream, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    laya::ck(cudaStreamEndCapture(g.stream, &graph), "end capture");
    if (p->dp.graph) cudaGraphExecDestroy(p->dp.graph);
    p->dp.graph = nullptr;
    cudaError_t ie = cudaGraphInstantiate(&p->dp.graph, graph, 0);
    cudaGraphDestroy(graph);
    laya::ck(ie, "graph instantiate");
    p->dp.graph_arena_gen = g.arena_gen;
    p->dp.launches = nl;
  });
}

int laya_plan_outputs(laya_engine* e, laya_plan* p, float* logits, float* act) {
  return guard([&] {
    if (!e || !p || !logits || !act) throw Error(LAYA_E_INVALID, "null argument");
    e->e->set_device();
    e->e->read_outputs(p->dp.host, logits, act);
  });
}

int laya_plan_stats(laya_plan* p, int64_t* real_tokens, int64_t* launches, int64_t* upload_bytes) {
  return guard([&] {
    if (!p) throw Error(LAYA_E_INVALID, "null plan");
    if (real_tokens) *real_tokens = p->dp.host.R;
    if (launches) *launches = p->dp.launches;
    if (upload_bytes) *upload_bytes = (int64_t)p->dp.lay.total;
  });
}

int laya_plan_profile(laya_engine* e, laya_plan* p, int steps, double* ms, int64_t* launches) {
  return guard([&] {
    if (!e || !p || !ms || !launches || steps <= 0) throw Error(LAYA_E_INVALID, "bad argument");
    Engine& g = *e->e;
    g.set_device();
    g.ensure_arena(p->dp.host);
    g.profile(p->dp, steps, ms, launches);
    g.check_device_error();
  });
}

void laya_plan_destroy(laya_plan* p) { delete p; }

int laya_plan_layout(const laya_req* req, int64_t* rows, int64_t* ntiles, int32_t* tiles, int64_t cap_tiles,
                     int64_t* nitems, int32_t* items, int64_t cap_items) {
  return guard([&] {
    if (!rows || !ntiles || !nitems) throw Error(LAYA_E_INVALID, "null argument");
    const laya::HostPlan p = laya::make_plan(req);
    *rows = p.R;
    *ntiles = p.ntiles;
    *nitems = p.nitems;
    if (tiles) {
      if (cap_tiles < p.ntiles) throw Error(LAYA_E_INVALID, "tile capacity too small");
      for (int i = 0; i < p.ntiles; ++i) {
        tiles[2 * i] = p.tiles[i].x;
        tiles[2 * i + 1] = p.tiles[i].y;
      }
    }
    if (items) {
      if (cap_items < p.nitems) throw Error(LAYA_E_INVALID, "item capacity too small");
      for (int i = 0; i < p.nitems; ++i) {
        items[4 * i] = p.items[i].x;
        items[4 * i + 1] = p.items[i].y;
        items[4 * i + 2] = p.items[i].z;
        items[4 * i + 3] = p.items[i].w;
      }
    }
  });
}

void* laya_stream(laya_engine* e) { return e ? (void*)e->e->stream : nullptr; }

int laya_plan_set_hidden(laya_engine* e, laya_plan* p, const float* x) {
  return guard([&] {
    if (!e || !p || !x) throw Error(LAYA_E_INVALID, "null argument");
    Engine& g = *e->e;
    g.set_device();
    g.ensure_arena(p->dp.host);
    laya::ck(cudaMemcpyAsync(g.x.p, x, (size_t)p->dp.host.R * laya::H * 4, cudaMemcpyHostToDevice, g.stream),
             "hidden upload");
    laya::ck(cudaStreamSynchronize(g.stream), "sync");
  });
}

int laya_plan_hidden(laya_engine* e, laya_plan* p, float* x) {
  return guard([&] {
    if (!e || !p || !x) throw Error(LAYA_E_INVALID, "null argument");
    Engine& g = *e->e;
    g.set_device();
    if (!g.x.p || g.cap_rows < p->dp.host.R) throw Error(LAYA_E_STATE, "no residual stream for this plan");
    laya::ck(cudaStreamSynchronize(g.stream), "sync");
    g.check_device_error();
    laya::ck(cudaMemcpy(x, g.x.p, (size_t)p->dp.host.R * laya::H * 4, cudaMemcpyDeviceToHost), "hidden download");
  });
}

int laya_plan_run_layer(laya_engine* e, laya_plan* p, int layer) {
  return guard([&] {
    if (!e || !p) throw Error(LAYA_E_INVALID, "null argument");
    if (layer < 0 || layer >= laya::NLAYER) throw Error(LAYA_E_INVALID, "layer out of range (0..27)");
    Engine& g = *e->e;
    g.set_device();
    g.ensure_arena(p->dp.host);
    g.enqueue_layer(p->dp, layer);
  });
}

int laya_selftest_gemm(int device, const uint16_t* a, const uint16_t* wt, float* out, int m, int n, int k,
                       int tile_n) {
  return guard([&] {
    if (tile_n != laya::kGemmBN && tile_n != laya::kGemmBNNarrow)
      throw Error(LAYA_E_INVALID, "selftest_gemm: tile_n must be 256 or 128");
    if (!a || !wt || !out || m <= 0 || n <= 0 || k <= 0 || n % tile_n || k % laya::kGemmBK)
      throw Error(LAYA_E_INVALID, "selftest_gemm: bad shape");
    laya::ck(cudaSetDevice(device), "cudaSetDevice");
    int sms = 0;
    laya::ck(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "attr");
    const int mp = (m + laya::kGemmBM - 1) / laya::kGemmBM * laya::kGemmBM;
    laya::DevBuf da, dw, dout, derr;
    da.alloc((size_t)mp * k * 2, "a");
    dw.alloc((size_t)n * k * 2, "w");
    dout.alloc((size_t)m * n * 4, "out");
    derr.alloc(256, "err");
    laya::ck(cudaMemset(da.p, 0, da.bytes), "memset");
    laya::ck(cudaMemset(derr.p, 0, 256), "memset");
    laya::ck(cudaMemcpy(da.p, a, (size_t)m * k * 2, cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(dw.p, wt, (size_t)n * k * 2, cudaMemcpyHostToDevice), "h2d");
    CUtensorMap ta, tw, to;
    if (laya::make_tmap_f16(&ta, da.p, m, k, laya::kGemmABoxRows) ||
        laya::make_tmap_f16(&tw, dw.p, n, k, tile_n / 2) ||
        laya::make_tmap_2d(&to, dout.p, true, m, n, 32, laya::kGemmOutBoxRows))
      throw Error(LAYA_E_CUDA, "tensor map encode failed");
    laya::GemmArgs g{};
    g.M = m;
    g.N = n;
    g.K = k;
    g.err = derr.as<int>();
    g.out = dout.p;
    g.ldo = n;
    laya::ck(laya::launch_gemm(laya::kEpiStoreF32, laya::GemmMaps{&ta, &tw, &to}, g, sms, 0, tile_n), "gemm launch");
    laya::ck(cudaDeviceSynchronize(), "gemm run");
    int ev = 0;
    laya::ck(cudaMemcpy(&ev, derr.p, 4, cudaMemcpyDeviceToHost), "d2h");
    if (ev) throw Error(LAYA_E_DEVICE_TIMEOUT, laya::fmt("gemm device wait expired (code %d)", ev));
    laya::ck(cudaMemcpy(out, dout.p, (size_t)m * n * 4, cudaMemcpyDeviceToHost), "d2h");
  });
}

int laya_bench_gemm(int device, int m, int n, int k, int tile_n, int epi, int flush_l2, int iters, float* ms) {
  return guard([&] {
    using namespace laya;
    const bool epi_ok = epi == kEpiQkvRope || epi == kEpiQkvBias || epi == kEpiResid || epi == kEpiGeglu ||
                        epi == kEpiBiasRelu || epi == kEpiStoreF32;
    if (!ms || m <= 0 || n <= 0 || k <= 0 || iters <= 0 || !epi_ok || (tile_n != kGemmBN && tile_n != kGemmBNNarrow) ||
        n % tile_n || k % kGemmBK || ((epi == kEpiQkvRope || epi == kEpiQkvBias) && n != 3 * H) ||
        (tile_n != kGemmBN && epi != kEpiResid && epi != kEpiStoreF32))
      throw Error(LAYA_E_INVALID, "bench_gemm: bad shape or epilogue");
    ck(cudaSetDevice(device), "cudaSetDevice");
    int sms = 0;
    ck(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "attr");
    const bool f32_out = epi == kEpiResid || epi == kEpiStoreF32;
    const int out_cols = epi == kEpiGeglu ? n / 2 : n;
    DevBuf da, dw, dout, derr, dpos, dcos, dsin, dbias, dflush;
    da.alloc((size_t)m * k * 2, "a");
    dw.alloc((size_t)n * k * 2, "w");
    dout.alloc((size_t)m * out_cols * (f32_out ? 4 : 2), "out");
    derr.alloc(256, "err");
    dpos.alloc((size_t)m * 4, "pos");
    dcos.alloc(128 * 32 * 4, "cos");
    dsin.alloc(128 * 32 * 4, "sin");
    dbias.alloc((size_t)n * 4, "bias");
    // operands: a fixed pattern (f16 1.0039 and 0.0655), no host copies
    ck(cudaMemset(da.p, 0x3c, da.bytes), "memset");
    ck(cudaMemset(dw.p, 0x2c, dw.bytes), "memset");
    ck(cudaMemset(dout.p, 0, dout.bytes), "memset");
    ck(cudaMemset(derr.p, 0, 256), "memset");
    ck(cudaMemset(dpos.p, 0, dpos.bytes), "memset");  // position 0 for every row
    ck(cudaMemset(dcos.p, 0, dcos.bytes), "memset");
    ck(cudaMemset(dsin.p, 0, dsin.bytes), "memset");
    ck(cudaMemset(dbias.p, 0, dbias.bytes), "memset");
    if (flush_l2) dflush.alloc((size_t)256 << 20, "l2 flush");
    CUtensorMap ta, tw, to;
    if (make_tmap_f16(&ta, da.p, m, k, kGemmABoxRows) || make_tmap_f16(&tw, dw.p, n, k, tile_n / 2) ||
        make_tmap_2d(&to, dout.p, f32_out, m, out_cols, f32_out ? 32 : 64, kGemmOutBoxRows))
      throw Error(LAYA_E_CUDA, "tensor map encode failed");
    GemmArgs g{};
    g.M = m;
    g.N = n;
    g.K = k;
    g.err = derr.as<int>();
    g.out = dout.p;
    g.ldo = out_cols;
    g.pos = dpos.as<int>();
    g.cosb = dcos.as<float>();
    g.sinb = dsin.as<float>();
    g.scale = 0.125f;
    g.bias = (epi == kEpiQkvBias || epi == kEpiBiasRelu) ? dbias.as<float>() : nullptr;
    g.n_valid = out_cols;
    const GemmMaps maps{&ta, &tw, &to};
    for (int i = 0; i < 3; ++i) ck(launch_gemm(epi, maps, g, sms, 0, tile_n), "gemm launch");
    std::vector<cudaEvent_t> ev(2 * (size_t)iters);
    for (auto& e : ev) ck(cudaEventCreate(&e), "event");
    for (int i = 0; i < iters; ++i) {
      if (flush_l2) ck(cudaMemsetAsync(dflush.p, i & 0xff, dflush.bytes, 0), "flush");
      ck(cudaEventRecord(ev[2 * i], 0), "event");
      ck(launch_gemm(epi, maps, g, sms, 0, tile_n), "gemm launch");
      ck(cudaEventRecord(ev[2 * i + 1], 0), "event");
    }
    ck(cudaEventSynchronize(ev.back()), "sync");
    float total = 0;
    for (int i = 0; i < iters; ++i) {
      float t = 0;
      ck(cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]), "elapsed");
      total += t;
    }
    for (auto e : ev) cudaEventDestroy(e);
    int errv = 0;
    ck(cudaMemcpy(&errv, derr.p, 4, cudaMemcpyDeviceToHost), "d2h");
    if (errv) throw Error(LAYA_E_DEVICE_TIMEOUT, fmt("gemm device wait expired (code %d)", errv));
    *ms = total / iters;
  });
}

int laya_test_timeout_next(laya_engine* e, int kind, uint64_t limit_ns) {
  return guard([&] {
    if (!e || (kind != 0 && kind != 1) || limit_ns == 0 || limit_ns > 2000000000ull)
      throw Error(LAYA_E_INVALID, "test_timeout_next: kind must be 0 or 1 and 0 < limit_ns <= 2e9");
    e->e->stuck_next = true;
    e->e->stuck_kind = kind;
    e->e->stuck_limit_ns = limit_ns;
  });
}

int laya_selftest_attention(int device, const uint16_t* qkv, const int32_t* lens, int n, int window, float* out,
                            int impl) {
  return guard([&] {
    if (!qkv || !lens || !out || n <= 0 || impl != 1)
      throw Error(LAYA_E_INVALID, "selftest_attention: bad argument (impl must be 1)");
    laya::ck(cudaSetDevice(device), "cudaSetDevice");
    int num_sms = 0;
    laya::ck(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device), "device query");
    std::vector<int> start(n), len(n);
    int R = 0;
    for (int b = 0; b < n; ++b) {
      if (lens[b] <= 0) throw Error(LAYA_E_INVALID, "selftest_attention: empty sequence");
      start[b] = R;
      len[b] = lens[b];
      R += lens[b];
    }
    std::vector<int2> tiles;
    std::vector<int4> items;
    laya::pack_short_tiles(start, len, 0, n, tiles);
    laya::attention_items(start, len, 0, n, items);
    std::vector<int> rowseq(R);
    for (int b = 0; b < n; ++b)
      for (int t = 0; t < len[b]; ++t) rowseq[start[b] + t] = b;
    laya::DevBuf dq, dout, dt, di, drs, ds, dl, derr;
    dq.alloc((size_t)R * 3072 * 2, "qkv");
    dout.alloc((size_t)R * 1024 * 2, "out");
    dt.alloc(std::max<size_t>(1, tiles.size()) * sizeof(int2), "tiles");
    di.alloc(std::max<size_t>(1, items.size()) * sizeof(int4), "items");
    drs.alloc((size_t)R * 4, "rowseq");
    ds.alloc((size_t)n * 4, "start");
    dl.alloc((size_t)n * 4, "len");
    laya::ck(cudaMemcpy(dq.p, qkv, dq.bytes, cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(dt.p, tiles.data(), tiles.size() * sizeof(int2), cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(di.p, items.data(), items.size() * sizeof(int4), cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(drs.p, rowseq.data(), (size_t)R * 4, cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(ds.p, start.data(), (size_t)n * 4, cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemcpy(dl.p, len.data(), (size_t)n * 4, cudaMemcpyHostToDevice), "h2d");
    laya::ck(cudaMemset(dout.p, 0, dout.bytes), "memset");
    derr.alloc(256, "err");
    laya::ck(cudaMemset(derr.p, 0, 256), "memset");
    CUtensorMap tm32;
    if (laya::make_tmap_2d(&tm32, dq.p, false, R, 3072, 64, laya::kAttnTcBoxRows))
      throw Error(LAYA_E_CUDA, "tensor map encode failed");
    laya::AttnShortArgs sa{};
    sa.out = dout.as<__half>();
    sa.tiles = dt.as<int2>();
    sa.rowseq = drs.as<int>();
    sa.seq_start = ds.as<int>();
    sa.seq_len = dl.as<int>();
    sa.num_tiles = (int)tiles.size();
    sa.window = window;
    sa.err = derr.as<int>();
    laya::ck(laya::launch_attention_short(&tm32, sa, num_sms, 0), "attention launch");
    laya::AttnArgs a{};
    a.out = dout.as<__half>();
    a.items = di.as<int4>();
    a.num_items = (int)items.size();
    a.window = window;
    a.err = derr.as<int>();
    laya::ck(laya::launch_attention_tc(&tm32, a, num_sms, 0), "attention launch");
    laya::ck(cudaDeviceSynchronize(), "attention run");
    int ev = 0;
    laya::ck(cudaMemcpy(&ev, derr.p, 4, cudaMemcpyDeviceToHost), "d2h");
    if (ev) throw Error(LAYA_E_DEVICE_TIMEOUT, laya::fmt("attention device wait expired (code %d)", ev));
    std::vector<uint16_t> h((size_t)R * 1024);
    laya::ck(cudaMemcpy(h.data(), dout.p, h.size() * 2, cudaMemcpyDeviceToHost), "d2h");
    for (size_t i = 0; i < h.size(); ++i) out[i] = laya::h2f_bits(h[i]);
  });
}

}  // extern "C"
