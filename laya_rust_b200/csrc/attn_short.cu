// Attention for sequences of at most 128 tokens on the 5th-generation tensor
// cores: a persistent, warp-specialised kernel that keeps four (tile, head)
// units in flight per SM.
//
// Contract (laya-rust backend/cpu/mod.rs:257-314 with the masks of
// :316-328): out = softmax(q . k^T + mask) . v per (sequence, head), q and k
// already scaled; a key is visible to a query of the same sequence and, on
// local layers, within +-window positions.
//
// A tile packs whole consecutive sequences of at most 128 tokens (adjacent
// in the compacted rows) into at most 128 rows; each row sees only its own
// sequence's keys, so packing changes no result and the tiles carry few
// padding rows.  A unit is (tile, head); unit u of the launch is tile u / 16,
// head u % 16, and CTA c (one per SM) takes a contiguous run of units, so
// the units it has in flight read adjacent column blocks of the same rows.
//
// Each CTA has four slots.  Slot s holds its units k = s, s + 4, ... (k
// counts this CTA's units): a shared-memory stage (Q | K | V, 16 KB each,
// 128-byte swizzle, only the 32-row boxes the tile's rows need) and 128 TMEM
// columns (S, then O over it).  Roles (608 threads):
//   warp 0      TMA producer: loads unit k into slot k % 4 as soon as the P.V
//               of unit k - 4 has completed (the stage is free)
//   warp 1      TMEM allocation; one thread issues S(k) = Q . K^T (M=128,
//               N=128, K=64) into the slot's TMEM once unit k is loaded and
//               the slot's TMEM is free
//   warp 2      one thread issues O(k) = P . [V | 1] (M=128, N=80, K=128)
//               over the dead S once the softmax has written P(k); two
//               issuers, so neither kind of step waits behind the other
//               The B operand of the second is V (64 columns) followed by an
//               all-ones block, so O's column 64 is the row sum of exactly
//               the f16 P values multiplied into V, summed on the tensor core.
//   warps 3-18  four softmax warpgroups, warpgroup s serving slot s: thread t
//               owns query row t = TMEM lane t.  It streams its scores from
//               TMEM 32 keys at a time (chunks no row of the warp sees get
//               no arithmetic, chunks every row of the warp sees fully take a
//               path without selects), takes the maximum, and writes
//               P = 2^(s log2 e - max) -- arguments rounded to f16 pairs, one
//               packed f16x2 exponential per two keys -- into the slot's dead
//               Q and K tiles (the swizzled K-major operand layout); after P.V
//               it scales its O row by 1 / sum and stores 64 f16 outputs,
//               then frees the slot's TMEM.
// So one slot's loads, another's MMAs and the softmax of the other two run
// at the same time, and no unit waits for a launch.
// Rows a tile does not use are never loaded: K rows past them are stale
// (their scores are masked), V rows past them hold an earlier unit's finite
// values or the zeros written at start (P is 0 there).
// Every wait is bounded; on expiry the thread records the error and raises
// the CTA's abort flag, every role leaves its loop, the MMA thread waits
// (bounded) for the MMAs it issued, the CTA lingers 2 ms so loads in flight
// land, and TMEM is freed.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int TQ = 128;
constexpr int D = 64;
constexpr int BOX = kAttnTcBoxRows;         // 32 rows per TMA box
constexpr int NSLOT = 4;
constexpr int CTRL_WARPS = 3;               // TMA producer, S issuer, P.V issuer
constexpr int SOFTMAX_WARPS = 4 * NSLOT;
constexpr int THREADS = 32 * (CTRL_WARPS + SOFTMAX_WARPS);
constexpr int TILE_BYTES = TQ * D * 2;      // 16 KB: one [128 x 64] f16 tile
constexpr int BOX_BYTES = BOX * D * 2;      // 4 KB
constexpr int STAGE_BYTES = 3 * TILE_BYTES; // Q | K | V
constexpr int DO = 80;                      // O columns: 64 outputs + the sum block
constexpr int OFF_ONES = NSLOT * STAGE_BYTES;          // all-ones [128 x 64] f16, after every V
constexpr int OFF_BAR = OFF_ONES + TILE_BYTES;
// barriers per slot: kv_full, s_full, p_full, o_full, tmem_free; then the
// two issuers' drains, stuck, the TMEM address and the abort flag
constexpr int NBARS = 5 * NSLOT + 3;
constexpr size_t SMEM = 1024 + OFF_BAR + NBARS * 8 + 16;
constexpr int TMEM_COLS = 512;              // slot s at column s * 128
constexpr float L2E = 1.4426950408889634f;

constexpr uint32_t IDESC_QK = umma_idesc_f16(TQ, TQ);
constexpr uint32_t IDESC_PV = umma_idesc_f16(TQ, DO) | (1u << 16);  // B ([V | 1]) MN-major

// MN-major operand written by TMA with 128-byte swizzle: rows are K (keys),
// 128 B of N (64 f16) per row, 8-row groups 1024 B apart (stride byte
// offset); the next 64 N columns start `lbo` bytes further (leading byte
// offset): here the all-ones block.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
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

// (x0 * inv, x1 * inv) of two f32 TMEM words in one packed multiply, as f16x2
// (x0 in the low half); each lane rounds as the scalar multiply.
__device__ __forceinline__ uint32_t scaled_h2(uint32_t x0, uint32_t x1, uint64_t inv2) {
  float p, q;
  f2_get(f2_mul(f2(u2f(x0), u2f(x1)), inv2), p, q);
  return pack_half2(p, q);
}

// (2^x0, 2^x1) as packed f16 (x0 in the low half): the arguments are
// rounded to f16 and one MUFU op exponentiates both.
__device__ __forceinline__ uint32_t exp2_h2(float x0, float x1) {
  uint32_t h, r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(h));
  return r;
}

__device__ __forceinline__ uint32_t tmem_ld_32x32b_x1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}

// Bits j of a 32-key chunk with a <= j < b (relative to the chunk).
__device__ __forceinline__ uint32_t chunk_mask(int a, int b) {
  const int lo = a < 0 ? 0 : (a > 32 ? 32 : a);
  const int hi = b < 0 ? 0 : (b > 32 ? 32 : b);
  if (hi <= lo) return 0u;
  const uint64_t m = ((1ull << hi) - 1ull) & ~((1ull << lo) - 1ull);
  return static_cast<uint32_t>(m);
}

// Running row maximum over one 32-key chunk of scores (4 partial maxima);
// `all`: every key of the chunk is visible to every row of the warp.
__device__ __forceinline__ void chunk_max(float (&mx)[4], const uint32_t (&v)[32], bool any, bool all,
                                          uint32_t mask) {
  if (!any) return;
  if (all) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) mx[(i >> 1) & 3] = fmax3f(mx[(i >> 1) & 3], u2f(v[i]), u2f(v[i + 1]));
  } else {
#pragma unroll
    for (int i = 0; i < 32; i += 2)
      mx[(i >> 1) & 3] = fmax3f(mx[(i >> 1) & 3], (mask >> i) & 1u ? u2f(v[i]) : -INFINITY,
                                (mask >> (i + 1)) & 1u ? u2f(v[i + 1]) : -INFINITY);
  }
}

// P = 2^(s log2 e - ms) of one 32-key chunk (0 for keys the row cannot see)
// into row r of the P operand: chunk ch -> K atom ch / 2 (the dead Q tile,
// then the dead K tile), 16-byte chunks 4 (ch % 2) .. of the row, swizzled.
__device__ __forceinline__ void chunk_p(uint8_t* st, int r, int ch, const uint32_t (&v)[32], bool any, bool all,
                                        uint32_t mask, float ms) {
  uint32_t w[16];
  if (!any) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0u;
  } else if (all) {
    // s log2 e - max for two keys per packed step
    const uint64_t l2e2 = f2_splat(L2E), nms2 = f2_splat(-ms);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float a0, a1;
      f2_get(f2_fma(f2(u2f(v[i]), u2f(v[i + 1])), l2e2, nms2), a0, a1);
      w[i / 2] = exp2_h2(a0, a1);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i += 2)
      w[i / 2] = exp2_h2((mask >> i) & 1u ? fmaf(u2f(v[i]), L2E, -ms) : -INFINITY,
                         (mask >> (i + 1)) & 1u ? fmaf(u2f(v[i + 1]), L2E, -ms) : -INFINITY);
  }
  uint8_t* prow = st + (ch >> 1) * TILE_BYTES + r * 128;
#pragma unroll
  for (int x = 0; x < 4; ++x)
    *reinterpret_cast<uint4*>(prow + (((4 * (ch & 1) + x) ^ (r & 7)) << 4)) =
        make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
}

// Lane 0 waits (bounded) and the warp agrees on the outcome; a warp that
// already failed does not wait again.
__device__ __forceinline__ bool warp_wait(bool ok, uint64_t* bar, uint32_t parity, const AttnShortArgs& a,
                                          volatile int* abort_flag) {
  int w = ok ? 1 : 0;
  if (ok && (threadIdx.x & 31) == 0)
    w = mbar_wait_bounded(bar, parity, a.err, kErrAttnWait, abort_flag, a.wait_limit_ns);
  return __shfl_sync(0xffffffffu, w, 0) != 0;
}

__device__ __forceinline__ int boxes_of(int rows) { return rows <= 0 ? 1 : (rows + BOX - 1) / BOX; }

__global__ void __launch_bounds__(THREADS, 1)
    attn_short_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ AttnShortArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* s_full = kv_full + NSLOT;
  uint64_t* p_full = s_full + NSLOT;
  uint64_t* o_full = p_full + NSLOT;
  uint64_t* tmem_free = o_full + NSLOT;
  uint64_t* drain = tmem_free + NSLOT;   // [2]: S issuer, P.V issuer
  uint64_t* stuck_bar = drain + 2;  // nothing ever arrives on it (the timeout test)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stuck_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // this CTA's units: a contiguous run [u0, u0 + my_units), so the units in
  // flight are adjacent heads of the same tile (neighbouring 128-byte column
  // blocks of the same q/k/v rows)
  const int total_units = a.num_tiles * 16;
  const int u0 = static_cast<int>((static_cast<long long>(blockIdx.x) * total_units) / gridDim.x);
  const int my_units =
      static_cast<int>((static_cast<long long>(blockIdx.x + 1) * total_units) / gridDim.x) - u0;

  if (tid == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);     // the four warps of the slot's warpgroup
      mbar_init(&o_full[s], 1);
      mbar_init(&tmem_free[s], 4);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    mbar_init(stuck_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
  }
  // V rows never loaded must be finite: zeros until a unit overwrites them;
  // the ones block feeds O's row-sum columns
  {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    const uint4 one = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);  // f16 1.0
    for (int i = tid; i < (NSLOT + 1) * TILE_BYTES / 16; i += THREADS) {
      const int s = i / (TILE_BYTES / 16), j = i - s * (TILE_BYTES / 16);
      if (s < NSLOT)
        reinterpret_cast<uint4*>(smem + s * STAGE_BYTES + 2 * TILE_BYTES)[j] = z;
      else
        reinterpret_cast<uint4*>(smem + OFF_ONES)[j] = one;
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the zeros, before the tensor core reads them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // the tiles come from the plan upload, which precedes every kernel of the
  // forward; q/k/v are written by the previous kernel
  grid_dep_wait();
  grid_dep_trigger();

  if (warp == 0) {
    // ---- TMA producer -------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      if (a.stuck) ok = mbar_wait_bounded(stuck_bar, 0, a.err, kErrAttnWait, abort_flag, a.wait_limit_ns);
      const uint64_t pol = l2_evict_first();  // q/k/v are read by this launch only
      int2 tile = my_units > 0 ? __ldg(a.tiles + (u0 >> 4)) : make_int2(0, 0);
      for (int k = 0; k < my_units && ok; ++k) {
        const int s = k % NSLOT, j = k / NSLOT;
        const int u = u0 + k;
        // the next unit's tile, in flight while this one waits for its slot
        const int2 tile_n = k + 1 < my_units ? __ldg(a.tiles + ((u + 1) >> 4)) : make_int2(0, 0);
        if (j > 0 && !(ok = mbar_wait_bounded(&o_full[s], (j - 1) & 1, a.err, kErrAttnWait, abort_flag,
                                              a.wait_limit_ns)))
          break;
        const int h = u & 15;
        const int nb = boxes_of(tile.y);
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&kv_full[s], 3 * nb * BOX_BYTES);
        for (int b = 0; b < nb; ++b) {
          tma_load_2d_hint(st + b * BOX_BYTES, &tm_qkv, h * D, tile.x + b * BOX, &kv_full[s], pol);
          tma_load_2d_hint(st + TILE_BYTES + b * BOX_BYTES, &tm_qkv, 1024 + h * D, tile.x + b * BOX, &kv_full[s],
                           pol);
          tma_load_2d_hint(st + 2 * TILE_BYTES + b * BOX_BYTES, &tm_qkv, 2048 + h * D, tile.x + b * BOX,
                           &kv_full[s], pol);
        }
        tile = tile_n;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---- S issuer: S(k) = Q . K^T once unit k is loaded and its slot's TMEM is free
    if (lane == 0) {
      bool ok = true;
      for (int k = 0; k < my_units && ok; ++k) {
        const int s = k % NSLOT, j = k / NSLOT;
        if (!(ok = mbar_wait_bounded(&kv_full[s], j & 1, a.err, kErrAttnWait, abort_flag, a.wait_limit_ns))) break;
        if (j > 0 &&
            !(ok = mbar_wait_bounded(&tmem_free[s], (j - 1) & 1, a.err, kErrAttnWait, abort_flag, a.wait_limit_ns)))
          break;
        tc_fence_after();
        uint8_t* st = smem + s * STAGE_BYTES;
        const uint64_t dq = umma_desc_sw128(smem_u32(st)), dk = umma_desc_sw128(smem_u32(st + TILE_BYTES));
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(s * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(d_tmem, dq + static_cast<uint64_t>(2 * kk), dk + static_cast<uint64_t>(2 * kk), IDESC_QK, kk > 0);
        umma_commit(&s_full[s]);
      }
      // every MMA issued here completes before TMEM is released
      umma_commit(&drain[0]);
      mbar_wait_bounded(&drain[0], 0, a.err, kErrAttnWait, nullptr);
    }
  } else if (warp == 2) {
    // ---- P.V issuer: O(k) = P . [V | 1] once the softmax has written P(k)
    if (lane == 0) {
      bool ok = true;
      const uint32_t ones = smem_u32(smem + OFF_ONES);
      for (int k = 0; k < my_units && ok; ++k) {
        const int s = k % NSLOT, j = k / NSLOT;
        if (!(ok = mbar_wait_bounded(&p_full[s], j & 1, a.err, kErrAttnWait, abort_flag, a.wait_limit_ns))) break;
        tc_fence_after();
        uint8_t* st = smem + s * STAGE_BYTES;
        const uint64_t dp = umma_desc_sw128(smem_u32(st));
        const uint32_t v_addr = smem_u32(st + 2 * TILE_BYTES);
        const uint64_t dv = desc_mn_sw128(v_addr, ones - v_addr);
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(s * 128);
#pragma unroll
        for (int kk = 0; kk < TQ / 16; ++kk)
          umma_f16(d_tmem, dp + static_cast<uint64_t>((kk >> 2) * (TILE_BYTES >> 4) + (kk & 3) * 2),
                   dv + static_cast<uint64_t>(kk * (2048 >> 4)), IDESC_PV, kk > 0);
        umma_commit(&o_full[s]);
      }
      umma_commit(&drain[1]);
      mbar_wait_bounded(&drain[1], 0, a.err, kErrAttnWait, nullptr);
    }
  } else {
    // ---- softmax warpgroup s ------------------------------------------------------
    const int s = (warp - CTRL_WARPS) >> 2;
    const int q = warp & 3;        // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;   // query row within the tile
    const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(s * 128);
    uint8_t* st = smem + s * STAGE_BYTES;
    bool ok = true;
    // The unit's tile and this row's visible keys [lo, hi) (tile-relative)
    // come from three dependent lookups (tile; row -> sequence; the
    // sequence's start and length).  They are pipelined one unit ahead: the
    // next unit's lookups are issued before this unit's softmax, after it
    // and before the P.V wait, so their latency hides behind the work.
    int2 tile = make_int2(0, 0);
    int lo = 0, hi = 0;
    if (s < my_units) {
      tile = __ldg(a.tiles + ((u0 + s) >> 4));
      if (r < tile.y) {
        const int sq = __ldg(a.rowseq + tile.x + r);
        const int sst = __ldg(a.seq_start + sq) - tile.x, en = sst + __ldg(a.seq_len + sq);
        lo = a.window >= 0 && r - a.window > sst ? r - a.window : sst;
        hi = a.window >= 0 && r + a.window + 1 < en ? r + a.window + 1 : en;
      }
    }
    for (int k = s, j = 0; k < my_units && ok; k += NSLOT, ++j) {
      const int u = u0 + k;
      const int h = u & 15;
      // lookup 1 of the next unit of this slot
      const bool has_next = k + NSLOT < my_units;
      const int2 tile_n = has_next ? __ldg(a.tiles + ((u + NSLOT) >> 4)) : make_int2(0, 0);
      if (!(ok = warp_wait(ok, &s_full[s], j & 1, a, abort_flag))) break;
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
        chunk_max(mx, v, true, all[ch], mask[ch]);
      }
      const float m = fmax3f(mx[0], mx[1], fmaxf(mx[2], mx[3]));
      const float ms = (m == -INFINITY ? 0.0f : m) * L2E;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + 32 * ch, v);
        tmem_ld_wait();
        chunk_p(st, r, ch, v, any[ch], all[ch], mask[ch], ms);
      }
      fence_proxy_async_smem();  // P, before the tensor core reads it
      tc_fence_before();         // S read before P.V overwrites it
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
      // lookups 2 and 3 of the next unit, in flight during the P.V wait and
      // the stores
      const bool real_n = r < tile_n.y;
      const int sq_n = real_n ? __ldg(a.rowseq + tile_n.x + r) : 0;
      const int st_n = real_n ? __ldg(a.seq_start + sq_n) : 0;
      const int len_n = real_n ? __ldg(a.seq_len + sq_n) : 0;
      if (!(ok = warp_wait(ok, &o_full[s], j & 1, a, abort_flag))) break;
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld_32x32b_x32(t_row, o0);
      tmem_ld_32x32b_x32(t_row + 32, o1);
      const float sum = u2f(tmem_ld_32x32b_x1(t_row + 64));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_free[s]);
      if (r < tile.y) {
        const uint64_t inv2 = f2_splat(sum > 0.0f ? 1.0f / sum : 0.0f);
        uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(tile.x + r) * 1024 + h * D);
#pragma unroll
        for (int x = 0; x < 4; ++x)
          dst[x] = make_uint4(scaled_h2(o0[8 * x], o0[8 * x + 1], inv2), scaled_h2(o0[8 * x + 2], o0[8 * x + 3], inv2),
                              scaled_h2(o0[8 * x + 4], o0[8 * x + 5], inv2),
                              scaled_h2(o0[8 * x + 6], o0[8 * x + 7], inv2));
#pragma unroll
        for (int x = 0; x < 4; ++x)
          dst[4 + x] = make_uint4(scaled_h2(o1[8 * x], o1[8 * x + 1], inv2),
                                  scaled_h2(o1[8 * x + 2], o1[8 * x + 3], inv2),
                                  scaled_h2(o1[8 * x + 4], o1[8 * x + 5], inv2),
                                  scaled_h2(o1[8 * x + 6], o1[8 * x + 7], inv2));
      }
      tile = tile_n;
      lo = hi = 0;
      if (real_n) {
        const int sst = st_n - tile_n.x, en = sst + len_n;
        lo = a.window >= 0 && r - a.window > sst ? r - a.window : sst;
        hi = a.window >= 0 && r + a.window + 1 < en ? r + a.window + 1 : en;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // a wait expired somewhere: loads already in flight land before teardown
    if (tid == 0) {
      const unsigned long long t0 = global_ns();
      while (global_ns() - t0 < 2000000ull) __nanosleep(1000);
    }
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_attention_short(const CUtensorMap* tm_qkv, const AttnShortArgs& a, int num_sms,
                                   cudaStream_t stream) {
  if (a.num_tiles <= 0) return cudaSuccess;
  if (!a.tiles || !a.rowseq || !a.seq_start || !a.seq_len || !a.out || !a.err || num_sms <= 0)
    return cudaErrorInvalidValue;
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
  const int units = a.num_tiles * 16;
  const int grid = units < num_sms ? units : num_sms;
  return launch_pdl(attn_short_kernel, dim3(grid), dim3(THREADS), SMEM, stream, nullptr, 0, *tm_qkv, a);
}

}  // namespace laya
