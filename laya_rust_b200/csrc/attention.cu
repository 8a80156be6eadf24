// Ragged flash attention over compacted sequences, f16 in / f32 softmax.
//
// Replaces the reference's materialised path (laya-rust
// src/backend/cuda/mod.rs:405-464: cuBLAS Q.K^T into an [n,16,l,l] f32 score
// buffer, k_add_mask, k_softmax, cuBLAS P.V, k_heads_to_seq) with one kernel.
// Semantics follow backend/cpu/mod.rs:257-314 with the mask of :316-328:
// a key t of sequence b is visible to query s when att[b,t] != 0 and, on local
// layers, |s - t| <= 64.  q and k arrive already scaled (the QKV epilogue
// applied SCALE to both), so scores are plain dot products.
//
// Layout: qkv is token-major [R, 3072] (q | k | v, head h at columns h*64);
// sequence b occupies rows [start[b], start[b] + len[b]).  The mask is a
// predicate on (len, window): no mask tensor exists.  Work that the mask
// removes is skipped, not computed: key blocks outside the CTA's band are
// never loaded, a warp whose 16 query rows lie past the sequence end does no
// math, and inside a key block each 16-key group that is past the end or
// outside the warp's +-64 band skips its QK^T and PV MMAs (its scores would
// be -inf and its probabilities 0, so the result is unchanged).
//
// CTA = 4 warps, 64 query rows (16 per warp) of one (sequence, head); keys in
// blocks of 64 through a 2-deep cp.async ring in XOR-swizzled shared memory;
// mma.sync m16n8k16 for S = Q.K^T and O += P.V with online softmax in
// registers.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int QR = kAttnQRows;
constexpr int KR = 64;
constexpr int D = 64;
constexpr int LDQKV = 3072;
constexpr float L2E = 1.4426950408889634f;

// element (r, c) of a [rows][64] f16 tile: 16-byte chunks XOR-swizzled by row
__device__ __forceinline__ int swz(int r, int c) { return r * D + ((((c >> 3) ^ (r & 7)) << 3) | (c & 7)); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = smem_u32(dst);
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Loads rows [row0, row0 + 64) of one 64-column slice of qkv into a swizzled
// tile; rows at or past `limit` are zero-filled.
__device__ __forceinline__ void load_tile(__half* tile, const __half* base, int row0, int limit, int col) {
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int r = i >> 3, ch = i & 7;
    const bool ok = row0 + r < limit;
    const __half* src = base + static_cast<size_t>(ok ? row0 + r : row0) * LDQKV + col + ch * 8;
    cp_async16(tile + swz(r, ch * 8), src, ok);
  }
}

__global__ void __launch_bounds__(128, 4) attention_kernel(const AttnArgs a) {
  __shared__ __align__(128) __half sQ[QR * D];
  __shared__ __align__(128) __half sK[2][KR * D];
  __shared__ __align__(128) __half sV[2][KR * D];

  const int2 blk = a.blocks[blockIdx.x];
  const int b = blk.x, q0 = blk.y, h = blockIdx.y;
  const int len = a.seq_len[b];
  const __half* base = a.qkv + static_cast<size_t>(a.seq_start[b]) * LDQKV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool windowed = a.window >= 0;

  // keys the whole CTA needs (union over its query rows)
  int k_lo = 0, k_hi = len;
  if (windowed) {
    k_lo = q0 - a.window;
    if (k_lo < 0) k_lo = 0;
    const int q_last = (q0 + QR < len ? q0 + QR : len) - 1;
    k_hi = q_last + a.window + 1;
    if (k_hi > len) k_hi = len;
  }
  const int kb0 = k_lo / KR;
  const int kb1 = (k_hi + KR - 1) / KR;

  // this warp's 16 query rows and the keys they can see
  const int qw0 = q0 + warp * 16;
  const bool warp_live = qw0 < len;
  int wk_lo = 0, wk_hi = len;
  if (windowed) {
    wk_lo = qw0 - a.window;
    if (wk_lo < 0) wk_lo = 0;
    wk_hi = qw0 + 15 + a.window + 1;
    if (wk_hi > len) wk_hi = len;
  }

  load_tile(sQ, base, q0, len, h * D);
  load_tile(sK[0], base, kb0 * KR, len, 1024 + h * D);
  load_tile(sV[0], base, kb0 * KR, len, 2048 + h * D);
  cp_commit();

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  uint32_t qf[4][4];
  const int qi0 = qw0 + g;  // this thread's two query rows: qi0, qi0 + 8

  for (int kb = kb0; kb < kb1; ++kb) {
    const int buf = (kb - kb0) & 1;
    if (kb + 1 < kb1) {
      load_tile(sK[buf ^ 1], base, (kb + 1) * KR, len, 1024 + h * D);
      load_tile(sV[buf ^ 1], base, (kb + 1) * KR, len, 2048 + h * D);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int key0 = kb * KR;
    // 16-key groups of this block that hold at least one key this warp sees
    bool live[4];
#pragma unroll
    for (int np = 0; np < 4; ++np) live[np] = warp_live && key0 + np * 16 < wk_hi && key0 + np * 16 + 16 > wk_lo;
    if (live[0] || live[1] || live[2] || live[3]) {
      if (kb == kb0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int m = lane >> 3;
          const int r = warp * 16 + (m & 1) * 8 + (lane & 7);
          const int c = kk * 16 + (m >> 1) * 8;
          ldsm_x4(qf[kk], sQ + swz(r, c));
        }
      }
      // S = Q . K^T for this warp's 16 rows x 64 keys
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
      const __half* tk = sK[buf];
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        if (!live[np]) continue;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int m = lane >> 3;
          const int r = np * 16 + (m >> 1) * 8 + (lane & 7);
          const int c = kk * 16 + (m & 1) * 8;
          uint32_t kf[4];
          ldsm_x4(kf, tk + swz(r, c));
          mma16816(s[2 * np], qf[kk], kf[0], kf[1]);
          mma16816(s[2 * np + 1], qf[kk], kf[2], kf[3]);
        }
      }
      // mask (only where this block crosses the sequence end or a band edge
      // of this warp's rows) + online softmax
      bool need_mask = key0 + KR > len;
      if (windowed) need_mask = need_mask || key0 < qw0 + 15 - a.window || key0 + KR - 1 > qw0 + a.window;
      float mx[2] = {-INFINITY, -INFINITY};
      if (need_mask) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int kidx = key0 + nt * 8 + 2 * t + (e & 1);
            const int qi = qi0 + (e >> 1) * 8;
            bool ok = live[nt >> 1] && kidx < len;
            if (windowed) {
              const int d = qi - kidx;
              ok = ok && d <= a.window && d >= -a.window;
            }
            const float v = ok ? s[nt][e] : -INFINITY;
            s[nt][e] = v;
            mx[e >> 1] = fmaxf(mx[e >> 1], v);
          }
        }
      } else {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
          mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
        }
      }
      float corr[2], m_use[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float m_new = fmaxf(m_run[r], mx[r]);
        m_use[r] = m_new == -INFINITY ? 0.0f : m_new;
        corr[r] = exp2f((m_run[r] - m_use[r]) * L2E);
        m_run[r] = m_new;
      }
      float rs[2] = {0.0f, 0.0f};
      uint32_t pf[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float p0 = exp2f((s[nt][0] - m_use[0]) * L2E);
        const float p1 = exp2f((s[nt][1] - m_use[0]) * L2E);
        const float p2 = exp2f((s[nt][2] - m_use[1]) * L2E);
        const float p3 = exp2f((s[nt][3] - m_use[1]) * L2E);
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        const int kk = nt >> 1;
        if ((nt & 1) == 0) {
          pf[kk][0] = pack2(p0, p1);
          pf[kk][1] = pack2(p2, p3);
        } else {
          pf[kk][2] = pack2(p0, p1);
          pf[kk][3] = pack2(p2, p3);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        o[dt][0] *= corr[0];
        o[dt][1] *= corr[0];
        o[dt][2] *= corr[1];
        o[dt][3] *= corr[1];
      }
      // O += P . V (16-key groups with no visible key have P = 0: skipped)
      const __half* tv = sV[buf];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (!live[kk]) continue;
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          const int m = lane >> 3;
          const int r = kk * 16 + (m & 1) * 8 + (lane & 7);
          const int c = dp * 16 + (m >> 1) * 8;
          uint32_t vf[4];
          ldsm_x4_t(vf, tv + swz(r, c));
          mma16816(o[2 * dp], pf[kk], vf[0], vf[1]);
          mma16816(o[2 * dp + 1], pf[kk], vf[2], vf[3]);
        }
      }
    } else if (kb == kb0 && warp_live) {
      // keep the Q fragments for later blocks of this warp
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int m = lane >> 3;
        const int r = warp * 16 + (m & 1) * 8 + (lane & 7);
        const int c = kk * 16 + (m >> 1) * 8;
        ldsm_x4(qf[kk], sQ + swz(r, c));
      }
    }
    __syncthreads();
  }

  if (!warp_live) return;
  float inv[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_run[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[r] = l > 0.0f ? 1.0f / l : 0.0f;
  }
  __half* out = a.out + static_cast<size_t>(a.seq_start[b]) * 1024 + h * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qi0 + r * 8;
    if (qi < len) {
      __half* orow = out + static_cast<size_t>(qi) * 1024;
#pragma unroll
      for (int dt = 0; dt < 8; ++dt)
        *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t) = pack2(o[dt][2 * r] * inv[r], o[dt][2 * r + 1] * inv[r]);
    }
  }
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, int num_blocks, cudaStream_t stream) {
  if (num_blocks == 0) return cudaSuccess;
  attention_kernel<<<dim3(num_blocks, 16), 128, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace laya
