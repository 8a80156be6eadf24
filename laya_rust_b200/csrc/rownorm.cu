// Row kernels: embedding gather + LayerNorm, LayerNorm (optionally gathered,
// or after adding a split-K GEMM's parts to the residual), and the final
// norm + type embedding + first head norm.  One warp per
// 1024-wide row, the row held in registers (32 values per lane), two-pass f32
// statistics, 512-byte coalesced loads and stores.
//
// Reference semantics: embedding (backend/cpu/mod.rs:145-153), layernorm
// (:155-186, eps 1e-5, weight-only on encoder layers, weight+bias in the head
// and scorer), add_type (:372-386), gather_markers (:388-398); graph order
// graph.rs:101-106 (layer 0 normalises the embedding and the normalised value
// seeds the residual stream, :113-114) and graph.rs:127-137.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int HID = 1024;
constexpr int ROWS_PER_CTA = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Normalises v[32] in place (weight/bias applied by the caller).
__device__ __forceinline__ void normalize(float (&v)[32], float eps) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) s += v[i];
  const float mean = warp_sum(s) * (1.0f / HID);
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
  const float var = warp_sum(q) * (1.0f / HID);
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = (v[i] - mean) * rstd;
}

// element index of v[4*i + j] held by `lane`: i*128 + lane*4 + j.  The rows
// are the residual stream, kept in L2 (evict-last) between the kernels that
// update and normalise it.
__device__ __forceinline__ void load_f32(const float* row, int lane, float (&v)[32]) {
  const float4* p = reinterpret_cast<const float4*>(row);
  const uint64_t pol = l2_evict_last();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 f;
    asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                 : "l"(p + i * 32 + lane), "l"(pol));
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
}

__device__ __forceinline__ void store_f32(float* row, int lane, const float (&v)[32]) {
  float4* p = reinterpret_cast<float4*>(row);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i * 32 + lane] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void store_f16(__half* row, int lane, const float (&v)[32]) {
  uint2* p = reinterpret_cast<uint2*>(row);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __half2 a = __floats2half2_rn(v[4 * i], v[4 * i + 1]);
    __half2 b = __floats2half2_rn(v[4 * i + 2], v[4 * i + 3]);
    p[i * 32 + lane] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
}

__device__ __forceinline__ void load_f16(const __half* row, int lane, float (&v)[32]) {
  const uint2* p = reinterpret_cast<const uint2*>(row);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint2 u = __ldg(p + i * 32 + lane);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = b.x; v[4 * i + 3] = b.y;
  }
}

__device__ __forceinline__ void scale_shift(float (&v)[32], int lane, const float* w, const float* b) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = __ldg(w4 + i * 32 + lane);
    v[4 * i] *= f.x; v[4 * i + 1] *= f.y; v[4 * i + 2] *= f.z; v[4 * i + 3] *= f.w;
  }
  if (b) {
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = __ldg(b4 + i * 32 + lane);
      v[4 * i] += f.x; v[4 * i + 1] += f.y; v[4 * i + 2] += f.z; v[4 * i + 3] += f.w;
    }
  }
}

// v += sum of the split-K parts of this row, the parts summed in part order
// first (so the result does not depend on which CTA finished first).  The
// parts are read once: streaming loads.
__device__ __forceinline__ void add_parts(float (&v)[32], const PendingParts& p, size_t row, int lane) {
  if (p.nparts <= 0 || row < static_cast<size_t>(p.row0)) return;
  row -= static_cast<size_t>(p.row0);
  float ps[32];
  const float4* q = reinterpret_cast<const float4*>(p.parts + row * HID);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = __ldcs(q + i * 32 + lane);
    ps[4 * i] = f.x; ps[4 * i + 1] = f.y; ps[4 * i + 2] = f.z; ps[4 * i + 3] = f.w;
  }
#pragma unroll 1
  for (int s = 1; s < p.nparts; ++s) {
    const float4* r = reinterpret_cast<const float4*>(p.parts + static_cast<size_t>(s) * p.stride + row * HID);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = __ldcs(r + i * 32 + lane);
      ps[4 * i] += f.x; ps[4 * i + 1] += f.y; ps[4 * i + 2] += f.z; ps[4 * i + 3] += f.w;
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += ps[i];
}

__global__ void __launch_bounds__(256) embed_ln_kernel(const __half* emb, const int* tok, const float* w,
                                                       float eps, float* x, __half* t16, int rows) {
  grid_dep_wait();
  grid_dep_trigger();
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[32];
  load_f16(emb + static_cast<size_t>(tok[row]) * HID, lane, v);
  normalize(v, eps);
  scale_shift(v, lane, w, nullptr);
  store_f32(x + static_cast<size_t>(row) * HID, lane, v);
  store_f16(t16 + static_cast<size_t>(row) * HID, lane, v);
}

__global__ void __launch_bounds__(256) ln_kernel(const float* x, const int* idx, const float* w, const float* b,
                                                 float eps, __half* t16, float* xo, int rows) {
  grid_dep_wait();
  grid_dep_trigger();
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int src = idx ? idx[row] : row;
  float v[32];
  load_f32(x + static_cast<size_t>(src) * HID, lane, v);
  normalize(v, eps);
  scale_shift(v, lane, w, b);
  if (xo) store_f32(xo + static_cast<size_t>(row) * HID, lane, v);
  store_f16(t16 + static_cast<size_t>(row) * HID, lane, v);
}

// A streaming 16-byte load kept in program order with the others (volatile),
// so a batch of them is in flight before the first sum needs one.
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) {
  float4 f;
  asm volatile("ld.global.cs.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w) : "l"(p));
  return f;
}

// add_parts with the part count known at compile time: the loads of G
// float4 chunks of every part are issued together (G * NP loads in flight
// per lane), then summed in add_parts' order, element by element.  The
// caller skips rows below p.row0 (they have no parts).
template <int NP>
__device__ __forceinline__ void add_parts_static(float (&v)[32], const PendingParts& p, size_t row, int lane) {
  row -= static_cast<size_t>(p.row0);
  constexpr int G = 32 / NP >= 8 ? 8 : 32 / NP;
  const float4* q = reinterpret_cast<const float4*>(p.parts + row * HID);
  const size_t st4 = p.stride / 4;
#pragma unroll
  for (int i0 = 0; i0 < 8; i0 += G) {
    float4 f[G][NP];
#pragma unroll
    for (int i = 0; i < G; ++i)
#pragma unroll
      for (int s = 0; s < NP; ++s)
        if (i0 + i < 8) f[i][s] = ld_stream_f4(q + s * st4 + (i0 + i) * 32 + lane);
#pragma unroll
    for (int i = 0; i < G; ++i) {
      if (i0 + i >= 8) continue;
      float4 a = f[i][0];
#pragma unroll
      for (int s = 1; s < NP; ++s) {
        a.x += f[i][s].x; a.y += f[i][s].y; a.z += f[i][s].z; a.w += f[i][s].w;
      }
      const int c = 4 * (i0 + i);
      v[c] += a.x; v[c + 1] += a.y; v[c + 2] += a.z; v[c + 3] += a.w;
    }
  }
}

// The residual add of a split-K GEMM (x += its NP parts) fused with the
// LayerNorm that follows it.  Rows below p.row0 have no parts: they are only
// normalised (their residual row is not rewritten).
template <int NP>
__global__ void __launch_bounds__(256) ln_parts_kernel(float* x, const PendingParts p, const float* w,
                                                       const float* b, float eps, __half* t16, int rows) {
  grid_dep_wait();
  grid_dep_trigger();
  // CTAs in reverse row order: the rows with parts (the last ones) read the
  // most and start first
  const int row = (gridDim.x - 1 - blockIdx.x) * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* xr = x + static_cast<size_t>(row) * HID;
  float v[32];
  load_f32(xr, lane, v);
  if (row >= p.row0) {
    add_parts_static<NP>(v, p, static_cast<size_t>(row), lane);
    store_f32(xr, lane, v);
  }
  normalize(v, eps);
  scale_shift(v, lane, w, b);
  store_f16(t16 + static_cast<size_t>(row) * HID, lane, v);
}

// x += parts alone, for a reader of the residual stream that is not a
// LayerNorm (taps, a single layer run on its own); the same arithmetic as
// ln_parts_kernel's first half.
__global__ void __launch_bounds__(256) add_parts_kernel(float* x, const PendingParts p, int rows) {
  grid_dep_wait();
  grid_dep_trigger();
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows || row < p.row0) return;  // rows below row0 have no parts
  float* xr = x + static_cast<size_t>(row) * HID;
  float v[32];
  load_f32(xr, lane, v);
  add_parts(v, p, static_cast<size_t>(row), lane);
  store_f32(xr, lane, v);
}

__global__ void __launch_bounds__(256) final_ln_kernel(float* x, const float* wf, const __half* type_emb,
                                                       const uint8_t* rowtype, const float* w1,
                                                       const float* b1, float eps, __half* t16,
                                                       int rows, const PendingParts p) {
  grid_dep_wait();
  grid_dep_trigger();
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* xr = x + static_cast<size_t>(row) * HID;
  float v[32], te[32];
  load_f32(xr, lane, v);
  add_parts(v, p, static_cast<size_t>(row), lane);
  normalize(v, eps);
  scale_shift(v, lane, wf, nullptr);
  load_f16(type_emb + static_cast<size_t>(rowtype[row]) * HID, lane, te);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += te[i];
  store_f32(xr, lane, v);
  normalize(v, eps);
  scale_shift(v, lane, w1, b1);
  store_f16(t16 + static_cast<size_t>(row) * HID, lane, v);
}

// ---- small batches: one 128-thread CTA per row ---------------------------------------
// With few rows the one-warp-per-row kernels run on few SMs and each warp
// walks a long dependent chain (the row, then its split-K parts).  Here a
// row's 1024 values are spread over 128 threads (two float4 each, 512-byte
// coalesced), so a 179-row batch keeps 179 SMs loading at once.  The
// arithmetic is the same as the warp kernels' (parts summed in part order,
// then added; two-pass f32 statistics), with the sums reduced over the block
// in a fixed order.
constexpr int kSmallRows = 1024;  // batches below this many rows take the per-row CTAs
constexpr int kRowThreads = 128;

// Sum over the CTA's 128 threads, the same value in every thread.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red is free (an earlier reduction has been read)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

template <int NP>
__global__ void __launch_bounds__(kRowThreads) ln_row_cta_kernel(float* x, const int* idx, const PendingParts p,
                                                                 const float* w, const float* b, float eps,
                                                                 __half* t16, int rows) {
  __shared__ float red[4];
  grid_dep_wait();
  grid_dep_trigger();
  const int row = blockIdx.x, t = threadIdx.x;
  if (row >= rows) return;
  const int src = idx ? idx[row] : row;
  float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(src) * HID);
  const uint64_t pol = l2_evict_last();
  float4 v[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v[i].x), "=f"(v[i].y), "=f"(v[i].z), "=f"(v[i].w)
                 : "l"(xr + t + 128 * i), "l"(pol));
  if constexpr (NP > 0) {
    if (row >= p.row0) {
      // parts summed in part order, then added (as add_parts)
      const float4* q = reinterpret_cast<const float4*>(p.parts + static_cast<size_t>(row - p.row0) * HID);
      const size_t st4 = p.stride / 4;
      float4 f[NP][2];
#pragma unroll
      for (int s = 0; s < NP; ++s)
#pragma unroll
        for (int i = 0; i < 2; ++i) f[s][i] = ld_stream_f4(q + s * st4 + t + 128 * i);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float4 a = f[0][i];
#pragma unroll
        for (int s = 1; s < NP; ++s) {
          a.x += f[s][i].x; a.y += f[s][i].y; a.z += f[s][i].z; a.w += f[s][i].w;
        }
        v[i].x += a.x; v[i].y += a.y; v[i].z += a.z; v[i].w += a.w;
        xr[t + 128 * i] = v[i];
      }
    }
  }
  const float mean = block_sum((v[0].x + v[0].y) + (v[0].z + v[0].w) + (v[1].x + v[1].y) + (v[1].z + v[1].w), red) *
                     (1.0f / HID);
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
    q += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
  }
  const float rstd = 1.0f / sqrtf(block_sum(q, red) * (1.0f / HID) + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  uint2* out = reinterpret_cast<uint2*>(t16 + static_cast<size_t>(row) * HID);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float4 g = __ldg(w4 + t + 128 * i);
    float4 y = make_float4((v[i].x - mean) * rstd * g.x, (v[i].y - mean) * rstd * g.y, (v[i].z - mean) * rstd * g.z,
                           (v[i].w - mean) * rstd * g.w);
    if (b) {
      const float4 c = __ldg(b4 + t + 128 * i);
      y.x += c.x; y.y += c.y; y.z += c.z; y.w += c.w;
    }
    const __half2 h0 = __floats2half2_rn(y.x, y.y), h1 = __floats2half2_rn(y.z, y.w);
    out[t + 128 * i] = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
  }
}

inline int grid_rows(int rows) { return (rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA; }

}  // namespace

cudaError_t launch_embed_ln(const __half* emb, const int* tok, const float* w, float eps, float* x,
                            __half* t16, int rows, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_pdl(embed_ln_kernel, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, emb, tok, w, eps, x, t16,
                    rows);
}

cudaError_t launch_ln(const float* x, const int* idx, const float* w, const float* b, float eps,
                      __half* t16, int rows, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (rows < kSmallRows)
    return launch_pdl(ln_row_cta_kernel<0>, dim3(rows), dim3(kRowThreads), 0, s, nullptr, 0, const_cast<float*>(x),
                      idx, PendingParts(), w, b, eps, t16, rows);
  return launch_pdl(ln_kernel, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, x, idx, w, b, eps, t16,
                    static_cast<float*>(nullptr), rows);
}

cudaError_t launch_ln_inplace(float* x, const float* w, float eps, __half* t16, int rows, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_pdl(ln_kernel, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, static_cast<const float*>(x),
                    static_cast<const int*>(nullptr), w, static_cast<const float*>(nullptr), eps, t16, x, rows);
}

template <int NP>
cudaError_t launch_ln_parts_n(float* x, const PendingParts& p, const float* w, const float* b, float eps,
                              __half* t16, int rows, cudaStream_t s) {
  if (rows < kSmallRows)
    return launch_pdl(ln_row_cta_kernel<NP>, dim3(rows), dim3(kRowThreads), 0, s, nullptr, 0, x,
                      static_cast<const int*>(nullptr), p, w, b, eps, t16, rows);
  return launch_pdl(ln_parts_kernel<NP>, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, x, p, w, b, eps, t16,
                    rows);
}

cudaError_t launch_ln_parts(float* x, const PendingParts& p, const float* w, const float* b, float eps,
                            __half* t16, int rows, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (!p.parts || p.nparts < 1 || p.row0 < 0 || p.stride < static_cast<size_t>(rows - p.row0) * HID || p.stride % 4)
    return cudaErrorInvalidValue;
  switch (p.nparts) {
    case 1: return launch_ln_parts_n<1>(x, p, w, b, eps, t16, rows, s);
    case 2: return launch_ln_parts_n<2>(x, p, w, b, eps, t16, rows, s);
    case 3: return launch_ln_parts_n<3>(x, p, w, b, eps, t16, rows, s);
    case 4: return launch_ln_parts_n<4>(x, p, w, b, eps, t16, rows, s);
    case 5: return launch_ln_parts_n<5>(x, p, w, b, eps, t16, rows, s);
    case 6: return launch_ln_parts_n<6>(x, p, w, b, eps, t16, rows, s);
    case 7: return launch_ln_parts_n<7>(x, p, w, b, eps, t16, rows, s);
    case 8: return launch_ln_parts_n<8>(x, p, w, b, eps, t16, rows, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_add_parts(float* x, const PendingParts& p, int rows, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (!p.parts || p.nparts < 1 || p.row0 < 0 || p.stride < static_cast<size_t>(rows - p.row0) * HID)
    return cudaErrorInvalidValue;
  return launch_pdl(add_parts_kernel, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, x, p, rows);
}

cudaError_t launch_final_ln(float* x, const float* wf, const __half* type_emb, const uint8_t* rowtype,
                            const float* w1, const float* b1, float eps, __half* t16, int rows,
                            cudaStream_t s, const PendingParts& p) {
  if (rows <= 0) return cudaSuccess;
  if (p.nparts > 0 && (!p.parts || p.row0 < 0 || p.stride < static_cast<size_t>(rows - p.row0) * HID))
    return cudaErrorInvalidValue;
  return launch_pdl(final_ln_kernel, dim3(grid_rows(rows)), dim3(256), 0, s, nullptr, 0, x, wf, type_emb, rowtype,
                    w1, b1, eps, t16, rows, p);
}

}  // namespace laya
