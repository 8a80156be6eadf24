// TEST / MEASUREMENT INFRASTRUCTURE ONLY: the reference's own GPU schedule,
// to time the reference's GPU algorithm on the same B200.  Nothing in the
// product links it.
//
// Restates the host side of laya-rust src/backend/cuda/mod.rs in C++: the
// buffer set of alloc (:154-189), ensure (:191-221, rope tables), mm / linear
// (:223-255, cuBLAS FP32 SGEMM in the default math mode), bmm_abt / bmm_ab
// (:257-301, strided-batched SGEMM), attention (:405-464: scores, add_mask,
// softmax, P.V, heads_to_seq) and forward (:466-812), launch shapes included
// (cfg = ceil(n/256) x 256, rows = one 256-thread block per row).  The device
// kernels are the reference's own CUDA source (src/backend/cuda/kernels.rs,
// the SRC string the reference compiles with NVRTC), extracted verbatim and
// compiled by oracle/ref_gpu_build.py into oracle/_ref/ (not committed); it
// is included here through REF_KERNELS.  Weights come from the C oracle's
// loaded model (f32, graph layout, as Tensors::f32 gives the reference).
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

#include REF_KERNELS

namespace {

constexpr int H = 1024, NH = 16, HD = 64, NLAYER = 28, INTER = 2624, WINDOW = 64, GLOBAL_EVERY = 3;
constexpr float EPS = 1e-5f, SCALE = 0.3535533845424652f;

thread_local std::string g_err;

struct Fail {
  std::string m;
};
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Fail{std::string(what) + ": " + cudaGetErrorString(e)};
}
void cb(cublasStatus_t e, const char* what) {
  if (e != CUBLAS_STATUS_SUCCESS) throw Fail{std::string(what) + ": cuBLAS status " + std::to_string(int(e))};
}
dim3 grid_cfg(size_t n) { return dim3(static_cast<unsigned>((n + 255) / 256 ? (n + 255) / 256 : 1)); }

struct Buf {
  void* p = nullptr;
  ~Buf() {
    if (p) cudaFree(p);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
  void alloc(size_t bytes) {
    if (p) cudaFree(p);
    p = nullptr;
    ck(cudaMalloc(&p, bytes ? bytes : 4), "cudaMalloc");
  }
};

struct Sched {
  int device = 0;
  cudaStream_t s = nullptr;
  cublasHandle_t blas = nullptr;
  std::map<std::string, Buf> w;
  size_t cn = 0, cl = 0, ck_ = 0;
  Buf x, t, qkv, q, kb, v, attn, ctx, p, mlp, gate, cos_a, sin_a, cos_b, sin_b, mask_g, mask_l, mrow, sc, logits,
      feats, aact, act, ids, att, mpos, mmask, qtype;

  const float* W(const std::string& n) const {
    auto it = w.find(n);
    if (it == w.end()) throw Fail{"weight " + n + " was not uploaded"};
    return it->second.as<float>();
  }

  // alloc (mod.rs:154-189) for the largest n, l, k seen, then the rope
  // tables (ensure, :191-221)
  void ensure(size_t n, size_t l, size_t k) {
    if (n <= cn && l <= cl && k <= ck_) return;
    cn = std::max(n, cn);
    cl = std::max(l, cl);
    ck_ = std::max(k, ck_);
    n = cn;
    l = cl;
    k = ck_;
    const size_t f = sizeof(float), i8 = sizeof(long long);
    x.alloc(n * l * H * f);
    t.alloc(n * std::max(l, k) * H * f);
    qkv.alloc(n * l * 3 * H * f);
    q.alloc(n * NH * l * HD * f);
    kb.alloc(n * NH * l * HD * f);
    v.alloc(n * NH * l * HD * f);
    attn.alloc(n * NH * l * l * f);
    ctx.alloc(n * l * H * f);
    p.alloc(n * l * H * f);
    mlp.alloc(std::max(n * l * 5248, n * k * H) * f);
    gate.alloc(n * l * INTER * f);
    for (Buf* b : {&cos_a, &sin_a, &cos_b, &sin_b}) b->alloc(l * 32 * f);
    mask_g.alloc(n * l * l * f);
    mask_l.alloc(n * l * l * f);
    mrow.alloc(n * k * H * f);
    sc.alloc(n * k * f);
    logits.alloc(n * k * f);
    feats.alloc(n * 4 * f);
    aact.alloc(n * (H + 4) * f);
    act.alloc(n * 2 * f);
    ids.alloc(n * l * i8);
    att.alloc(n * l * i8);
    mpos.alloc(n * k * i8);
    mmask.alloc(n * k * i8);
    qtype.alloc(n * i8);
    const int seq = static_cast<int>(l), half = 32;
    k_rope_table<<<grid_cfg(l * 32), 256, 0, s>>>(W("rope.freq_full"), cos_a.as<float>(), sin_a.as<float>(), seq, half);
    k_rope_table<<<grid_cfg(l * 32), 256, 0, s>>>(W("rope.freq_sliding"), cos_b.as<float>(), sin_b.as<float>(), seq,
                                                  half);
    ck(cudaGetLastError(), "rope");
  }

  // mm: x [m,k] . W [k,n] (graph layout), column-major view (mod.rs:223-238)
  void mm(const float* a, const float* wt, float* c, int m, int n, int k) {
    const float one = 1.f, zero = 0.f;
    cb(cublasSgemm(blas, CUBLAS_OP_N, CUBLAS_OP_N, n, m, k, &one, wt, n, a, k, &zero, c, n), "mm");
  }
  // linear: x [m,k] . W[n,k]^T (mod.rs:240-255)
  void linear(const float* a, const float* wt, float* c, int m, int n, int k) {
    const float one = 1.f, zero = 0.f;
    cb(cublasSgemm(blas, CUBLAS_OP_T, CUBLAS_OP_N, n, m, k, &one, wt, k, a, k, &zero, c, n), "linear");
  }
  void layernorm(const float* xi, const float* wt, const float* bias, float* y, size_t rows) {
    k_layernorm<<<static_cast<unsigned>(rows), 256, 0, s>>>(xi, wt, bias, y, H, EPS);
  }
  void add(float* a, const float* b, size_t n) { k_add<<<grid_cfg(n), 256, 0, s>>>(a, b, static_cast<long long>(n)); }
  void add_bias(float* xi, const float* b, int dim, size_t n) {
    k_add_bias<<<grid_cfg(n), 256, 0, s>>>(xi, b, dim, static_cast<long long>(n));
  }
  void split_qkv(const float* cs, const float* sn, size_t n, size_t l, int rope) {
    const size_t total = n * NH * l * HD;
    k_split_qkv<<<grid_cfg(total), 256, 0, s>>>(qkv.as<float>(), cs, sn, q.as<float>(), kb.as<float>(), v.as<float>(),
                                                static_cast<long long>(total), static_cast<int>(l), NH, HD, SCALE,
                                                rope);
  }
  // attention (mod.rs:405-464)
  void attention(const float* mask, size_t n, size_t l) {
    const int li = static_cast<int>(l), batch = static_cast<int>(n * NH);
    const float one = 1.f, zero = 0.f;
    // bmm_abt(q, k, attn, batch, l, l, HD): the A operand is k, B is q
    cb(cublasSgemmStridedBatched(blas, CUBLAS_OP_T, CUBLAS_OP_N, li, li, HD, &one, kb.as<float>(), HD,
                                 static_cast<long long>(l) * HD, q.as<float>(), HD, static_cast<long long>(l) * HD,
                                 &zero, attn.as<float>(), li, static_cast<long long>(l) * l, batch),
       "bmm_abt");
    const size_t total = n * NH * l * l;
    k_add_mask<<<grid_cfg(total), 256, 0, s>>>(attn.as<float>(), mask, static_cast<long long>(total), li, NH);
    k_softmax<<<static_cast<unsigned>(n * NH * l), 256, 0, s>>>(attn.as<float>(), li);
    // bmm_ab(attn, v, q, batch, l, HD, l): the A operand is v, B is attn
    cb(cublasSgemmStridedBatched(blas, CUBLAS_OP_N, CUBLAS_OP_N, HD, li, li, &one, v.as<float>(), HD,
                                 static_cast<long long>(l) * HD, attn.as<float>(), li, static_cast<long long>(l) * l,
                                 &zero, q.as<float>(), HD, static_cast<long long>(l) * HD, batch),
       "bmm_ab");
    const size_t t2 = n * NH * l * HD;
    k_heads_to_seq<<<grid_cfg(t2), 256, 0, s>>>(q.as<float>(), ctx.as<float>(), static_cast<long long>(t2), li, NH,
                                                HD);
  }

  // forward (mod.rs:466-812)
  void forward(size_t n, size_t l, size_t k, const int64_t* hids, const int64_t* hatt, const int64_t* hmpos,
               const int64_t* hmmask, const int64_t* hqtype, float* out_logits, float* out_act) {
    ensure(n, l, k);
    const size_t nl = n * l;
    const int hi = H, li = static_cast<int>(l), ki = static_cast<int>(k);
    ck(cudaMemcpyAsync(ids.p, hids, nl * 8, cudaMemcpyHostToDevice, s), "h2d");
    ck(cudaMemcpyAsync(att.p, hatt, nl * 8, cudaMemcpyHostToDevice, s), "h2d");
    ck(cudaMemcpyAsync(mpos.p, hmpos, n * k * 8, cudaMemcpyHostToDevice, s), "h2d");
    ck(cudaMemcpyAsync(mmask.p, hmmask, n * k * 8, cudaMemcpyHostToDevice, s), "h2d");
    ck(cudaMemcpyAsync(qtype.p, hqtype, n * 8, cudaMemcpyHostToDevice, s), "h2d");
    k_gather_rows<<<static_cast<unsigned>(nl), 256, 0, s>>>(ids.as<long long>(),
                                                             W("encoder.embeddings.tok_embeddings.weight"),
                                                             x.as<float>(), hi);
    const dim3 mg(static_cast<unsigned>((l + 255) / 256 ? (l + 255) / 256 : 1), static_cast<unsigned>(l),
                  static_cast<unsigned>(n));
    k_mask_build<<<mg, 256, 0, s>>>(att.as<long long>(), mask_g.as<float>(), li, 0);
    k_mask_build<<<mg, 256, 0, s>>>(att.as<long long>(), mask_l.as<float>(), li, WINDOW);
    char nm[96];
    for (int layer = 0; layer < NLAYER; ++layer) {
      const bool global = layer % GLOBAL_EVERY == 0;
      if (layer == 0) snprintf(nm, sizeof nm, "encoder.embeddings.norm.weight");
      else snprintf(nm, sizeof nm, "encoder.layers.%d.attn_norm.weight", layer);
      layernorm(x.as<float>(), W(nm), nullptr, t.as<float>(), nl);
      snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wqkv.weight", layer);
      mm(t.as<float>(), W(nm), qkv.as<float>(), static_cast<int>(nl), 3 * hi, hi);
      split_qkv(global ? cos_a.as<float>() : cos_b.as<float>(), global ? sin_a.as<float>() : sin_b.as<float>(), n, l,
                1);
      attention(global ? mask_g.as<float>() : mask_l.as<float>(), n, l);
      snprintf(nm, sizeof nm, "encoder.layers.%d.attn.Wo.weight", layer);
      mm(ctx.as<float>(), W(nm), p.as<float>(), static_cast<int>(nl), hi, hi);
      if (layer == 0)
        k_copy<<<grid_cfg(nl * H), 256, 0, s>>>(x.as<float>(), t.as<float>(), static_cast<long long>(nl * H));
      add(x.as<float>(), p.as<float>(), nl * H);
      snprintf(nm, sizeof nm, "encoder.layers.%d.mlp_norm.weight", layer);
      layernorm(x.as<float>(), W(nm), nullptr, t.as<float>(), nl);
      snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wi.weight", layer);
      mm(t.as<float>(), W(nm), mlp.as<float>(), static_cast<int>(nl), 5248, hi);
      k_gelu_mul<<<grid_cfg(nl * INTER), 256, 0, s>>>(mlp.as<float>(), gate.as<float>(), static_cast<long long>(nl),
                                                      static_cast<long long>(INTER));
      snprintf(nm, sizeof nm, "encoder.layers.%d.mlp.Wo.weight", layer);
      mm(gate.as<float>(), W(nm), p.as<float>(), static_cast<int>(nl), hi, INTER);
      add(x.as<float>(), p.as<float>(), nl * H);
    }
    layernorm(x.as<float>(), W("encoder.final_norm.weight"), nullptr, t.as<float>(), nl);
    k_copy<<<grid_cfg(nl * H), 256, 0, s>>>(x.as<float>(), t.as<float>(), static_cast<long long>(nl * H));
    k_add_type<<<grid_cfg(nl * H), 256, 0, s>>>(x.as<float>(), W("type_emb.weight"), qtype.as<long long>(),
                                                static_cast<long long>(nl * H), li, hi);
    for (int layer = 0; layer < 2; ++layer) {
      auto hn = [&](const char* suf) {
        snprintf(nm, sizeof nm, "head.layers.%d.%s", layer, suf);
        return W(nm);
      };
      layernorm(x.as<float>(), hn("norm1.weight"), hn("norm1.bias"), t.as<float>(), nl);
      mm(t.as<float>(), hn("self_attn.in_proj_weight"), qkv.as<float>(), static_cast<int>(nl), 3 * hi, hi);
      add_bias(qkv.as<float>(), hn("self_attn.in_proj_bias"), 3 * H, nl * 3 * H);
      split_qkv(cos_a.as<float>(), cos_a.as<float>(), n, l, 0);
      attention(mask_g.as<float>(), n, l);
      linear(ctx.as<float>(), hn("self_attn.out_proj.weight"), p.as<float>(), static_cast<int>(nl), hi, hi);
      add_bias(p.as<float>(), hn("self_attn.out_proj.bias"), H, nl * H);
      add(x.as<float>(), p.as<float>(), nl * H);
      layernorm(x.as<float>(), hn("norm2.weight"), hn("norm2.bias"), t.as<float>(), nl);
      mm(t.as<float>(), hn("linear1.weight"), mlp.as<float>(), static_cast<int>(nl), 4096, hi);
      add_bias(mlp.as<float>(), hn("linear1.bias"), 4096, nl * 4096);
      k_relu<<<grid_cfg(nl * 4096), 256, 0, s>>>(mlp.as<float>(), static_cast<long long>(nl * 4096));
      mm(mlp.as<float>(), hn("linear2.weight"), p.as<float>(), static_cast<int>(nl), hi, 4096);
      add_bias(p.as<float>(), hn("linear2.bias"), H, nl * H);
      add(x.as<float>(), p.as<float>(), nl * H);
    }
    k_marker_gather<<<static_cast<unsigned>(n * k), 256, 0, s>>>(x.as<float>(), mpos.as<long long>(),
                                                                  mrow.as<float>(), li, ki, hi);
    layernorm(mrow.as<float>(), W("scorer.0.weight"), W("scorer.0.bias"), t.as<float>(), n * k);
    mm(t.as<float>(), W("scorer.1.weight"), mlp.as<float>(), static_cast<int>(n * k), hi, hi);
    add_bias(mlp.as<float>(), W("scorer.1.bias"), H, n * k * H);
    k_gelu<<<grid_cfg(n * k * H), 256, 0, s>>>(mlp.as<float>(), static_cast<long long>(n * k * H));
    mm(mlp.as<float>(), W("scorer.3.weight"), sc.as<float>(), static_cast<int>(n * k), 1, hi);
    add_bias(sc.as<float>(), W("scorer.3.bias"), 1, n * k);
    k_post<<<static_cast<unsigned>(n), 256, k * 4, s>>>(sc.as<float>(), mmask.as<long long>(), logits.as<float>(),
                                                        feats.as<float>(), ki);
    k_act_input<<<grid_cfg(n * (H + 4)), 256, 0, s>>>(x.as<float>(), feats.as<float>(), aact.as<float>(),
                                                      static_cast<long long>(n * (H + 4)), li, hi, 4);
    linear(aact.as<float>(), W("act_head.0.weight"), p.as<float>(), static_cast<int>(n), 256, H + 4);
    add_bias(p.as<float>(), W("act_head.0.bias"), 256, n * 256);
    k_gelu<<<grid_cfg(n * 256), 256, 0, s>>>(p.as<float>(), static_cast<long long>(n * 256));
    linear(p.as<float>(), W("act_head.2.weight"), act.as<float>(), static_cast<int>(n), 2, 256);
    add_bias(act.as<float>(), W("act_head.2.bias"), 2, n * 2);
    ck(cudaGetLastError(), "kernel launch");
    if (out_logits) ck(cudaMemcpyAsync(out_logits, logits.p, n * k * 4, cudaMemcpyDeviceToHost, s), "d2h");
    if (out_act) ck(cudaMemcpyAsync(out_act, act.p, n * 2 * 4, cudaMemcpyDeviceToHost, s), "d2h");
    ck(cudaStreamSynchronize(s), "forward");
  }
};

template <class F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const Fail& e) {
    g_err = e.m;
    return 1;
  }
}

}  // namespace

extern "C" {

const char* rg_error(void) { return g_err.c_str(); }

void* rg_open(int device) {
  auto* g = new Sched();
  if (guard([&] {
        g->device = device;
        ck(cudaSetDevice(device), "cudaSetDevice");
        ck(cudaStreamCreateWithFlags(&g->s, cudaStreamNonBlocking), "stream");
        cb(cublasCreate(&g->blas), "cublasCreate");
        cb(cublasSetStream(g->blas, g->s), "cublasSetStream");
      })) {
    delete g;
    return nullptr;
  }
  return g;
}

int rg_upload(void* h, const char* name, const float* data, size_t count) {
  auto* g = static_cast<Sched*>(h);
  return guard([&] {
    ck(cudaSetDevice(g->device), "cudaSetDevice");
    Buf& b = g->w[name];
    b.alloc(count * 4);
    ck(cudaMemcpy(b.p, data, count * 4, cudaMemcpyHostToDevice), "weight upload");
  });
}

int rg_forward(void* h, int64_t n, int64_t l, int64_t k, const int64_t* ids, const int64_t* att, const int64_t* mpos,
               const int64_t* mmask, const int64_t* qtype, float* logits, float* act) {
  auto* g = static_cast<Sched*>(h);
  return guard([&] {
    ck(cudaSetDevice(g->device), "cudaSetDevice");
    g->forward(n, l, k, ids, att, mpos, mmask, qtype, logits, act);
  });
}

// Mean device time of `iters` forwards (CUDA events on the schedule's
// stream around each; request copies included, as the reference's forward
// does them).
int rg_time(void* h, int64_t n, int64_t l, int64_t k, const int64_t* ids, const int64_t* att, const int64_t* mpos,
            const int64_t* mmask, const int64_t* qtype, int iters, float* ms) {
  auto* g = static_cast<Sched*>(h);
  return guard([&] {
    ck(cudaSetDevice(g->device), "cudaSetDevice");
    g->forward(n, l, k, ids, att, mpos, mmask, qtype, nullptr, nullptr);
    cudaEvent_t e0, e1;
    ck(cudaEventCreate(&e0), "event");
    ck(cudaEventCreate(&e1), "event");
    float total = 0.f;
    for (int i = 0; i < iters; ++i) {
      ck(cudaEventRecord(e0, g->s), "event");
      g->forward(n, l, k, ids, att, mpos, mmask, qtype, nullptr, nullptr);
      ck(cudaEventRecord(e1, g->s), "event");
      ck(cudaEventSynchronize(e1), "event");
      float t = 0.f;
      ck(cudaEventElapsedTime(&t, e0, e1), "elapsed");
      total += t;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms = total / iters;
  });
}

void rg_close(void* h) {
  auto* g = static_cast<Sched*>(h);
  if (!g) return;
  cudaSetDevice(g->device);
  if (g->s) cudaStreamSynchronize(g->s);
  g->w.clear();
  if (g->blas) cublasDestroy(g->blas);
  if (g->s) cudaStreamDestroy(g->s);
  delete g;
}

}  // extern "C"
