// Attention for sequences of at most 128 tokens on the 5th-generation tensor
// cores: one CTA per (tile, head), a single pass.
//
// Contract (laya-rust backend/cpu/mod.rs:257-314 with the masks of
// :316-328): out = softmax(q . k^T + mask) . v per (sequence, head), q and k
// already scaled; a key is visible to a query of the same sequence and, on
// local layers, within +-window positions.
//
// A tile packs whole consecutive sequences of at most 128 tokens (adjacent
// in the compacted rows) into at most 128 rows; each row sees only its own
// sequence's keys, so packing changes no result and the tiles carry few
// padding rows.  Per CTA (128 threads, 48 KB shared memory, 128 TMEM
// columns: four CTAs per SM):
//   TMA      Q, K, V [128 rows x 64] of one head from the token-major qkv
//            buffer, 128-byte swizzle
//   MMA 1    S = Q . K^T -> TMEM columns [0, 128)     (M=128, N=128, K=64)
//   softmax  thread t owns query row t = TMEM lane t: its visible keys are an
//            interval; it streams its scores from TMEM 32 keys at a time
//            (chunks no row of the warp sees are skipped, chunks every row of
//            the warp sees fully take a path without selects), takes the
//            maximum, then writes P = exp(s - max) as f16 into shared memory
//            over the dead Q and K tiles (the swizzled K-major operand layout)
//            and sums it
//   MMA 2    O = P . V -> TMEM columns [0, 64) over the dead S (M=128, N=64,
//            K=128), V as an MN-major operand
//   store    thread t scales its O row by 1 / sum and writes 64 f16
// Every wait is bounded; a CTA whose wait expires records the error, lets
// the operations it issued land and returns.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int TQ = 128;
constexpr int D = 64;
constexpr int THREADS = 128;
constexpr int TILE_BYTES = TQ * D * 2;  // 16 KB: one [128 x 64] f16 tile
constexpr int TMEM_COLS = 128;
constexpr size_t SMEM = 1024 + 3 * TILE_BYTES + 64;  // + barriers kv, s, o, stuck, drain and the TMEM address
constexpr float L2E = 1.4426950408889634f;

constexpr uint32_t IDESC_QK = umma_idesc_f16(TQ, TQ);
constexpr uint32_t IDESC_PV = umma_idesc_f16(TQ, D) | (1u << 16);  // B (V) MN-major

// MN-major operand written by TMA with 128-byte swizzle: rows are K (keys),
// 128 B of N (64 f16) per row, 8-row groups 1024 B apart; one N block.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(TILE_BYTES >> 4) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bits j of a 32-key chunk with a <= j < b (relative to the chunk).
__device__ __forceinline__ uint32_t chunk_mask(int a, int b) {
  const int lo = a < 0 ? 0 : (a > 32 ? 32 : a);
  const int hi = b < 0 ? 0 : (b > 32 ? 32 : b);
  if (hi <= lo) return 0u;
  const uint64_t m = ((1ull << hi) - 1ull) & ~((1ull << lo) - 1ull);
  return static_cast<uint32_t>(m);
}

__global__ void __launch_bounds__(THREADS, 4)
    attn_short_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ AttnShortArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;                   // then P, over Q and K
  uint8_t* sK = smem + TILE_BYTES;
  uint8_t* sV = smem + 2 * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * TILE_BYTES);
  uint64_t* kv_bar = bars;
  uint64_t* s_bar = bars + 1;
  uint64_t* o_bar = bars + 2;
  uint64_t* stuck_bar = bars + 3;  // nothing ever arrives on it (the timeout test)
  uint64_t* drain = bars + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 5);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int2 tile = a.tiles[blockIdx.x];  // (first row, rows); uploaded before every kernel of the forward
  const int h = blockIdx.y;
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  grid_dep_wait();
  grid_dep_trigger();

  bool ok = true;
  if (tid == 0) {
    if (a.stuck) ok = mbar_wait_bounded(stuck_bar, 0, a.err, kErrAttnWait, nullptr, a.wait_limit_ns);
    if (ok) {
      const uint64_t pol = l2_evict_first();
      mbar_arrive_expect_tx(kv_bar, 3 * TILE_BYTES);
      tma_load_2d_hint(sQ, &tm_qkv, h * D, tile.x, kv_bar, pol);
      tma_load_2d_hint(sK, &tm_qkv, 1024 + h * D, tile.x, kv_bar, pol);
      tma_load_2d_hint(sV, &tm_qkv, 2048 + h * D, tile.x, kv_bar, pol);
    }
  }
  // the query row of this thread and its visible keys (tile-relative)
  const int r = tid;
  int lo = 0, hi = 0;
  if (r < tile.y) {
    const int s = a.rowseq[tile.x + r];
    const int st = a.seq_start[s] - tile.x, en = st + a.seq_len[s];
    lo = a.window >= 0 && r - a.window > st ? r - a.window : st;
    hi = a.window >= 0 && r + a.window + 1 < en ? r + a.window + 1 : en;
  }
  if (__syncthreads_or(!ok)) ok = false;
  if (ok) ok = mbar_wait_bounded(kv_bar, 0, a.err, kErrAttnWait, nullptr, a.wait_limit_ns);
  if (__syncthreads_or(!ok)) ok = false;

  // S = Q . K^T
  if (ok && tid == 0) {
    tc_fence_after();
    const uint64_t dq = umma_desc_sw128(smem_u32(sQ)), dk = umma_desc_sw128(smem_u32(sK));
#pragma unroll
    for (int k = 0; k < D / 16; ++k)
      umma_f16(tmem, dq + static_cast<uint64_t>(2 * k), dk + static_cast<uint64_t>(2 * k), IDESC_QK, k > 0);
    umma_commit(s_bar);
  }
  if (ok) ok = mbar_wait_bounded(s_bar, 0, a.err, kErrAttnWait, nullptr, a.wait_limit_ns);
  if (__syncthreads_or(!ok)) ok = false;

  const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float sum = 0.0f;
  if (ok) {
    tc_fence_after();
    uint32_t mask[4];
    bool any[4], all[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      mask[ch] = chunk_mask(lo - 32 * ch, hi - 32 * ch);
      any[ch] = __any_sync(0xffffffffu, mask[ch] != 0u);
      all[ch] = __all_sync(0xffffffffu, mask[ch] == 0xffffffffu);
    }
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      if (!any[ch]) continue;
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + 32 * ch, v);
      tmem_ld_wait();
      if (all[ch]) {
#pragma unroll
        for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], u2f(v[j]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], (mask[ch] >> j) & 1u ? u2f(v[j]) : -INFINITY);
      }
    }
    const float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
    const float ms = (m == -INFINITY ? 0.0f : m) * L2E;
    float sm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t w[16];
      if (!any[ch]) {
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = 0u;
      } else {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + 32 * ch, v);
        tmem_ld_wait();
        float p[32];
        if (all[ch]) {
#pragma unroll
          for (int j = 0; j < 32; ++j) p[j] = fast_exp2(fmaf(u2f(v[j]), L2E, -ms));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            p[j] = fast_exp2((mask[ch] >> j) & 1u ? fmaf(u2f(v[j]), L2E, -ms) : -INFINITY);
        }
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          sm[(j >> 1) & 3] += p[j] + p[j + 1];
          w[j / 2] = pack_half2(p[j], p[j + 1]);
        }
      }
      // chunk ch -> K atom ch / 2 (16 KB apart), 16-byte chunks 4 (ch % 2) ..
      uint8_t* prow = sQ + (ch >> 1) * TILE_BYTES + r * 128;
#pragma unroll
      for (int x = 0; x < 4; ++x)
        *reinterpret_cast<uint4*>(prow + (((4 * (ch & 1) + x) ^ (r & 7)) << 4)) =
            make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
    }
    sum = (sm[0] + sm[1]) + (sm[2] + sm[3]);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  if (__syncthreads_or(!ok)) ok = false;  // P complete, S read by all

  // O = P . V over the dead S columns
  if (ok && tid == 0) {
    tc_fence_after();
    const uint64_t dp = umma_desc_sw128(smem_u32(sQ));
    const uint64_t dv = desc_mn_sw128(smem_u32(sV));
#pragma unroll
    for (int kk = 0; kk < TQ / 16; ++kk)
      umma_f16(tmem, dp + static_cast<uint64_t>((kk >> 2) * (TILE_BYTES >> 4) + (kk & 3) * 2),
               dv + static_cast<uint64_t>(kk * (2048 >> 4)), IDESC_PV, kk > 0);
    umma_commit(o_bar);
  }
  if (ok) ok = mbar_wait_bounded(o_bar, 0, a.err, kErrAttnWait, nullptr, a.wait_limit_ns);
  if (__syncthreads_or(!ok)) ok = false;
  if (ok) {
    tc_fence_after();
    uint32_t o0[32], o1[32];
    tmem_ld_32x32b_x32(t_row, o0);
    tmem_ld_32x32b_x32(t_row + 32, o1);
    tmem_ld_wait();
    if (r < tile.y) {
      const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
      uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(tile.x + r) * 1024 + h * D);
#pragma unroll
      for (int x = 0; x < 4; ++x)
        dst[x] = make_uint4(pack_half2(u2f(o0[8 * x]) * inv, u2f(o0[8 * x + 1]) * inv),
                            pack_half2(u2f(o0[8 * x + 2]) * inv, u2f(o0[8 * x + 3]) * inv),
                            pack_half2(u2f(o0[8 * x + 4]) * inv, u2f(o0[8 * x + 5]) * inv),
                            pack_half2(u2f(o0[8 * x + 6]) * inv, u2f(o0[8 * x + 7]) * inv));
#pragma unroll
      for (int x = 0; x < 4; ++x)
        dst[4 + x] = make_uint4(pack_half2(u2f(o1[8 * x]) * inv, u2f(o1[8 * x + 1]) * inv),
                                pack_half2(u2f(o1[8 * x + 2]) * inv, u2f(o1[8 * x + 3]) * inv),
                                pack_half2(u2f(o1[8 * x + 4]) * inv, u2f(o1[8 * x + 5]) * inv),
                                pack_half2(u2f(o1[8 * x + 6]) * inv, u2f(o1[8 * x + 7]) * inv));
    }
  } else if (tid == 0) {
    // a wait expired: MMAs and loads already issued land before teardown
    umma_commit(drain);
    mbar_wait_bounded(drain, 0, a.err, kErrAttnWait, nullptr, 0);
    const unsigned long long t0 = global_ns();
    while (global_ns() - t0 < 2000000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_attention_short(const CUtensorMap* tm_qkv, const AttnShortArgs& a, cudaStream_t stream) {
  if (a.num_tiles <= 0) return cudaSuccess;
  if (!a.tiles || !a.rowseq || !a.seq_start || !a.seq_len || !a.out || !a.err) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(attn_short_kernel, dim3(a.num_tiles, 16), dim3(THREADS), SMEM, stream, nullptr, 0, *tm_qkv, a);
}

}  // namespace laya
