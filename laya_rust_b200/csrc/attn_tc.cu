// Ragged attention on the 5th-generation tensor cores (tcgen05 + TMEM):
// a persistent, warp-specialised flash kernel with an online softmax.
//
// Contract (laya-rust backend/cpu/mod.rs:257-314 with the masks of
// :316-328): out = softmax(q . k^T + mask) . v per (sequence, head), q and k
// already scaled; a key is visible to a query when it is a real token of
// the same sequence and, on local layers, within +-window positions.  No
// mask tensor exists: each query row derives its visible key interval
// [lo, hi) from its sequence's row span and the window.
//
// Work: a unit is (item, head); an item is 128 query rows of the compacted
// batch with the key blocks they can see.  Items are either a tile of whole
// consecutive sequences of at most 128 tokens (one key block: the tile
// itself) or a 128-row block of a longer sequence (1-4 key blocks of 128,
// those outside the window skipped).  One CTA per SM walks the units
// blockIdx.x, blockIdx.x + gridDim.x, ...; unit k of a CTA goes to slot
// k & 1, so two units are in flight per CTA and one slot's softmax overlaps
// the other slot's MMAs and loads.
//
// Roles (320 threads):
//   warp 0      TMA producer: Q of each unit into the slot's Q buffer, then
//               its K and V blocks into a 3-stage ring (32 KB per stage)
//   warp 1      TMEM allocation; one thread issues the MMAs:
//                 S[slot] = Q . K_j^T        (M=128, N=128, K=64) -> TMEM
//                 O[slot] += P_j . V_j       (M=128, N=64,  K=128) -> TMEM
//               in a fixed order shared with the producer (the two slots'
//               key-block steps alternate; each S is followed by the P.V of
//               the step before it)
//   warps 2-5   softmax warpgroup of slot 0, warps 6-9 of slot 1: thread t
//               owns query row t = TMEM lane t.  Per key block it reads its
//               128 scores, takes the running maximum, writes
//               P = exp(s - max) as f16 into the slot's P buffer (the
//               swizzled K-major operand layout), rescales its O row in TMEM
//               when the maximum grew, and accumulates the row sum; after
//               the unit's last block it scales O by 1 / sum and stores the
//               row's 64 f16 values.
// Shared memory: Q 2 x 16 KB, K/V ring 3 x 32 KB, P 2 x 32 KB (193 KB).
// TMEM: S 2 x 128 columns, O 2 x 64 columns (512 allocated).
//
// Every wait is bounded (2 s by default).  On expiry the waiting thread
// records an error code and raises the CTA's abort flag; every role leaves
// its loop at its next wait, the MMA thread waits (bounded) for the MMAs it
// issued, the CTA lingers 2 ms so TMA loads in flight land, and TMEM is
// freed.  The host reads the error word after the forward.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int TQ = 128;                  // query rows per item
constexpr int TK = 128;                  // keys per block
constexpr int D = 64;                    // head dim
constexpr int NKV = 3;                   // K/V ring stages
constexpr int THREADS = 320;
constexpr int TILE_BYTES = TQ * D * 2;   // 16 KB: one [128 x 64] f16 tile
constexpr int KV_BYTES = 2 * TILE_BYTES; // K then V
constexpr int P_BYTES = 2 * TILE_BYTES;  // P [128 x 128] f16: two 64-key atoms
constexpr int OFF_Q = 0;
constexpr int OFF_KV = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_P = OFF_KV + NKV * KV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
// barriers: q_full[2] q_empty[2] kv_full[NKV] kv_empty[NKV] s_full[2]
// p_full[2] pv_done[2] drain stuck, then the TMEM address and the abort flag
constexpr int NBARS = 2 + 2 + NKV + NKV + 2 + 2 + 2 + 2;
constexpr size_t SMEM = 1024 + OFF_BAR + NBARS * 8 + 16;
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0;                 // S[slot] at slot * 128
constexpr int O_COL = 256;               // O[slot] at 256 + slot * 64
constexpr float L2E = 1.4426950408889634f;

// S: A = Q (K-major), B = K block (K-major), M = 128, N = 128
constexpr uint32_t IDESC_QK = umma_idesc_f16(TQ, TK);
// O: A = P (K-major over keys), B = V (MN-major: d contiguous), M = 128, N = 64
constexpr uint32_t IDESC_PV = umma_idesc_f16(TQ, D) | (1u << 16);

// Descriptor of an MN-major operand tile written by TMA with 128-byte
// swizzle: rows are K (keys), 128 B of N (64 f16) per row; 8-row groups
// 1024 B apart (stride byte offset); a single 64-wide N block.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(TILE_BYTES >> 4) << 16;  // next N block (unused: N = 64)
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

// 2^x with the hardware approximation (relative error ~2^-22): one MUFU op.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bits j of a 32-key chunk with a <= j < b (a, b relative to the chunk, any
// integers): the keys of the chunk one query row can see.
__device__ __forceinline__ uint32_t chunk_mask(int a, int b) {
  const int lo = a < 0 ? 0 : (a > 32 ? 32 : a);
  const int hi = b < 0 ? 0 : (b > 32 ? 32 : b);
  if (hi <= lo) return 0u;
  const uint64_t m = ((1ull << hi) - 1ull) & ~((1ull << lo) - 1ull);
  return static_cast<uint32_t>(m);
}

// The key blocks a unit's queries can see: [kb0, kb1) of 128 keys counted
// from the sequence's first row (windowed on local layers).
struct ItemGeom {
  int q_row0, q_rows, k_row0, nkb;
};

__device__ __forceinline__ ItemGeom item_geom(const int4 it, int window) {
  // it = (first query row, query rows, sequence start row, sequence length);
  // a tile of packed short sequences has start = first row, length = rows
  const int q0 = it.x - it.z, len = it.w;
  int lo = 0, hi = len;
  if (window >= 0) {
    lo = q0 - window > 0 ? q0 - window : 0;
    hi = q0 + it.y + window < len ? q0 + it.y + window : len;
  }
  const int kb0 = lo / TK, kb1 = (hi + TK - 1) / TK;
  return ItemGeom{it.x, it.y, it.z + kb0 * TK, kb1 - kb0};
}

// The fixed order of key-block steps shared by the producer and the MMA
// thread: the two slots' steps alternate (a slot whose units are exhausted
// drops out).  Slot s holds this CTA's units k = s, s + 2, ...
struct StepIter {
  const AttnArgs* a;
  int units;                 // units of this CTA
  int k[2], j[2], nkb[2], n[2];
  int turn;
  __device__ __forceinline__ void load(int s) {
    if (k[s] < units) {
      const int u = blockIdx.x + k[s] * gridDim.x;
      nkb[s] = item_geom(a->items[u >> 4], a->window).nkb;
      if (nkb[s] <= 0) nkb[s] = 1;  // never: every item has a key block
    }
  }
  __device__ __forceinline__ void init(const AttnArgs* args, int cta_units) {
    a = args;
    units = cta_units;
    k[0] = 0; k[1] = 1; j[0] = j[1] = 0; n[0] = n[1] = 0; turn = 0;
    load(0);
    load(1);
  }
  // Next step: slot, unit index k within the CTA, block j, its unit's block
  // count and the slot's running step count c.  False when both are done.
  __device__ __forceinline__ bool next(int& slot, int& kk, int& jj, int& nb, int& c) {
    int s = turn;
    if (k[s] >= units) s ^= 1;
    if (k[s] >= units) return false;
    slot = s; kk = k[s]; jj = j[s]; nb = nkb[s]; c = n[s];
    ++n[s];
    if (++j[s] == nkb[s]) {
      j[s] = 0;
      k[s] += 2;
      load(s);
    }
    turn = s ^ 1;
    return true;
  }
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const AttnArgs& a, int code,
                                         volatile int* abort_flag) {
  return mbar_wait_bounded(bar, parity, a.err, code, abort_flag, a.wait_limit_ns);
}

__global__ void __launch_bounds__(THREADS, 1)
    attn_flash_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + NKV;
  uint64_t* s_full = kv_empty + NKV;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* drain = pv_done + 2;
  uint64_t* stuck_bar = drain + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stuck_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total_units = a.num_items * 16;
  const int my_units = blockIdx.x < total_units ? (total_units - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(stuck_bar, 1);  // nothing ever arrives on it (the timeout test)
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  grid_dep_wait();
  grid_dep_trigger();

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      if (a.stuck) ok = wait_bar(stuck_bar, 0, a, kErrAttnWait, abort_flag);
      const uint64_t pol = l2_evict_first();  // q/k/v are read by this launch only
      StepIter it;
      it.init(&a, my_units);
      uint32_t qe_phase[2] = {0, 0}, kve_phase = 0;
      int nq[2] = {0, 0}, stage = 0;
      int slot, kk, jj, nb, c;
      while (ok && it.next(slot, kk, jj, nb, c)) {
        const int u = blockIdx.x + kk * gridDim.x;
        const int h = u & 15;
        const ItemGeom g = item_geom(a.items[u >> 4], a.window);
        if (jj == 0) {
          if (nq[slot] > 0) {
            if (!(ok = wait_bar(&q_empty[slot], qe_phase[slot], a, kErrAttnWait, abort_flag))) break;
            qe_phase[slot] ^= 1u;
          }
          ++nq[slot];
          mbar_arrive_expect_tx(&q_full[slot], TILE_BYTES);
          tma_load_2d_hint(smem + OFF_Q + slot * TILE_BYTES, &tm_qkv, h * D, g.q_row0, &q_full[slot], pol);
        }
        if (!(ok = wait_bar(&kv_empty[stage], kve_phase ^ 1u, a, kErrAttnWait, abort_flag))) break;
        uint8_t* kv = smem + OFF_KV + stage * KV_BYTES;
        const int krow = g.k_row0 + jj * TK;
        mbar_arrive_expect_tx(&kv_full[stage], KV_BYTES);
        tma_load_2d_hint(kv, &tm_qkv, 1024 + h * D, krow, &kv_full[stage], pol);
        tma_load_2d_hint(kv + TILE_BYTES, &tm_qkv, 2048 + h * D, krow, &kv_full[stage], pol);
        if (++stage == NKV) {
          stage = 0;
          kve_phase ^= 1u;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      StepIter it;
      it.init(&a, my_units);
      uint32_t qf_phase[2] = {0, 0}, kvf_phase = 0, pf_phase[2] = {0, 0};
      int p_seen[2] = {0, 0};  // p_full completions consumed per slot
      int stage = 0;
      // the step issued last, whose P.V follows the next S
      bool pend = false;
      int pend_slot = 0, pend_stage = 0, pend_c = 0;
      bool pend_first = false;
      auto wait_p = [&](int s, int count) {
        while (ok && p_seen[s] < count) {
          ok = wait_bar(&p_full[s], pf_phase[s], a, kErrAttnWait, abort_flag);
          pf_phase[s] ^= 1u;
          ++p_seen[s];
        }
        return ok;
      };
      auto issue_pv = [&]() {
        // P_j of the pending step is written (and its O rescaled) once p_full
        // completes for the slot's (c + 1)-th time
        if (!wait_p(pend_slot, pend_c + 1)) return;
        tc_fence_after();
        const uint32_t pa = smem_u32(smem + OFF_P + pend_slot * P_BYTES);
        const uint32_t va = smem_u32(smem + OFF_KV + pend_stage * KV_BYTES + TILE_BYTES);
        const uint32_t d = tmem + O_COL + pend_slot * D;
#pragma unroll
        for (int kk2 = 0; kk2 < TK / 16; ++kk2)
          umma_f16(d, umma_desc_sw128(pa + (kk2 >> 2) * TILE_BYTES + (kk2 & 3) * 32),
                   desc_mn_sw128(va + kk2 * 2048), IDESC_PV, (!pend_first || kk2 > 0) ? 1u : 0u);
        umma_commit(&kv_empty[pend_stage]);
        umma_commit(&pv_done[pend_slot]);
        pend = false;
      };
      int slot, kk, jj, nb, c;
      while (ok && it.next(slot, kk, jj, nb, c)) {
        // S[slot] is free once the slot's previous step has its P written
        if (!wait_p(slot, c)) break;
        if (jj == 0) {
          if (!(ok = wait_bar(&q_full[slot], qf_phase[slot], a, kErrAttnWait, abort_flag))) break;
          qf_phase[slot] ^= 1u;
        }
        if (!(ok = wait_bar(&kv_full[stage], kvf_phase, a, kErrAttnWait, abort_flag))) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + OFF_Q + slot * TILE_BYTES);
        const uint32_t ka = smem_u32(smem + OFF_KV + stage * KV_BYTES);
#pragma unroll
        for (int k4 = 0; k4 < D / 16; ++k4)
          umma_f16(tmem + S_COL + slot * TK, umma_desc_sw128(qa + k4 * 32), umma_desc_sw128(ka + k4 * 32), IDESC_QK,
                   k4 > 0 ? 1u : 0u);
        umma_commit(&s_full[slot]);
        if (jj == nb - 1) umma_commit(&q_empty[slot]);
        if (pend) {
          issue_pv();
          if (!ok) break;
        }
        pend = true;
        pend_slot = slot;
        pend_stage = stage;
        pend_c = c;
        pend_first = jj == 0;
        if (++stage == NKV) {
          stage = 0;
          kvf_phase ^= 1u;
        }
      }
      if (ok && pend) issue_pv();
      if (!ok) *abort_flag = 1;
      // every MMA issued here completes before TMEM is released
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, a.err, kErrAttnWait, nullptr, 0);
    }
  } else {
    // ---- softmax warpgroups --------------------------------------------------------
    const int slot = (warp - 2) >> 2;
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    const int row = q * 32 + lane;              // query row within the item
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t t_s = t_lane + S_COL + slot * TK;
    const uint32_t t_o = t_lane + O_COL + slot * D;
    uint8_t* prow = smem + OFF_P + slot * P_BYTES + row * 128;
    uint32_t sf_phase = 0, pv_phase = 0;
    bool ok = true;
    for (int kk = slot; kk < my_units && ok; kk += 2) {
      const int u = blockIdx.x + kk * gridDim.x;
      const int h = u & 15;
      const ItemGeom g = item_geom(a.items[u >> 4], a.window);
      const bool valid = row < g.q_rows;
      const int r_abs = g.q_row0 + row;
      int lo = 0, hi = 0;  // visible keys, absolute rows
      if (valid) {
        const int2 sp = a.rowspan[r_abs];
        lo = sp.x;
        hi = sp.y;
        if (a.window >= 0) {
          lo = r_abs - a.window > lo ? r_abs - a.window : lo;
          hi = r_abs + a.window + 1 < hi ? r_abs + a.window + 1 : hi;
        }
      }
      float m_run = -INFINITY, l_run = 0.0f;
      for (int jj = 0; jj < g.nkb && ok; ++jj) {
        int w_ok = 1;
        if (lane == 0) w_ok = wait_bar(&s_full[slot], sf_phase, a, kErrAttnWait, abort_flag);
        sf_phase ^= 1u;
        if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // keys [a, b) of this block are visible to the row (block-relative)
        const int kbase = g.k_row0 + jj * TK;
        const int a0 = lo - kbase, b0 = hi - kbase;
        // pass 1: block maximum, streaming S from TMEM 32 keys at a time;
        // a chunk no row of the warp can see is skipped (warp-uniformly)
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          const uint32_t mask = chunk_mask(a0 - 32 * ch, b0 - 32 * ch);
          if (!__any_sync(0xffffffffu, mask != 0u)) continue;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_s + 32 * ch, v);
          tmem_ld_wait();
          if (__all_sync(0xffffffffu, mask == 0xffffffffu)) {
#pragma unroll
            for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], u2f(v[j]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], (mask >> j) & 1u ? u2f(v[j]) : -INFINITY);
          }
        }
        const float mb = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float m_new = fmaxf(m_run, mb);
        const float m_use = m_new == -INFINITY ? 0.0f : m_new;
        const float ms = m_use * L2E;
        // O and l were accumulated against m_run: rescale by 2^((m_run - m_new) log2 e)
        const float alpha = m_run == -INFINITY ? 0.0f : fast_exp2((m_run - m_use) * L2E);
        // the slot's previous P.V must be done: P is rewritten and O rescaled
        if (jj > 0) {
          int v_ok = 1;
          if (lane == 0) v_ok = wait_bar(&pv_done[slot], pv_phase, a, kErrAttnWait, abort_flag);
          pv_phase ^= 1u;
          if (!__shfl_sync(0xffffffffu, v_ok, 0)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        // pass 2: P = 2^(s log2e - max) (0 where hidden) as f16 into this
        // row of P (chunk ch -> K atom ch / 2, 16-byte chunks 4 (ch % 2) ..)
        float sm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          const uint32_t mask = chunk_mask(a0 - 32 * ch, b0 - 32 * ch);
          uint32_t w[16];
          if (!__any_sync(0xffffffffu, mask != 0u)) {
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = 0u;
          } else {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_s + 32 * ch, v);
            tmem_ld_wait();
            float p[32];
            if (__all_sync(0xffffffffu, mask == 0xffffffffu)) {
#pragma unroll
              for (int j = 0; j < 32; ++j) p[j] = fast_exp2(fmaf(u2f(v[j]), L2E, -ms));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                p[j] = fast_exp2((mask >> j) & 1u ? fmaf(u2f(v[j]), L2E, -ms) : -INFINITY);
            }
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              sm[(j >> 1) & 3] += p[j] + p[j + 1];
              w[j / 2] = pack_half2(p[j], p[j + 1]);
            }
          }
          uint8_t* pr = prow + (ch >> 1) * TILE_BYTES;
          const int c0 = (ch & 1) * 4;
#pragma unroll
          for (int x = 0; x < 4; ++x)
            *reinterpret_cast<uint4*>(pr + (((c0 + x) ^ (row & 7)) << 4)) =
                make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
        }
        const float sum = (sm[0] + sm[1]) + (sm[2] + sm[3]);
        l_run = jj == 0 ? sum : l_run * alpha + sum;
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows' maximum grew (alpha is 1 elsewhere)
        if (jj > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
          uint32_t o[32];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            tmem_ld_32x32b_x32(t_o + 32 * hh, o);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(u2f(o[j]) * alpha);
            tmem_st_32x32b_x32(t_o + 32 * hh, o);
          }
          tmem_st_wait();
        }
        m_run = m_new;
        fence_proxy_async_smem();  // P (generic writes) visible to the tensor core
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[slot]);
      }
      if (!ok) break;
      // the unit's last P.V, then the epilogue
      int v_ok = 1;
      if (lane == 0) v_ok = wait_bar(&pv_done[slot], pv_phase, a, kErrAttnWait, abort_flag);
      pv_phase ^= 1u;
      if (!__shfl_sync(0xffffffffu, v_ok, 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld_32x32b_x32(t_o, o0);
      tmem_ld_32x32b_x32(t_o + 32, o1);
      tmem_ld_wait();
      if (valid) {
        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(r_abs) * 1024 + h * D);
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
      tc_fence_before();  // O read before the slot's next unit overwrites it
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && tid == 0) {
    // a wait expired: TMA loads issued before the abort land before the CTA
    // (and its shared memory) goes away
    const unsigned long long t0 = global_ns();
    while (global_ns() - t0 < 2000000ull) __nanosleep(1000);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_attention_tc(const CUtensorMap* tm_qkv, const AttnArgs& a, int num_sms, cudaStream_t stream) {
  if (a.num_items <= 0) return cudaSuccess;
  if (!a.items || !a.rowspan || !a.out || !a.err || num_sms <= 0) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attn_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const long long units = static_cast<long long>(a.num_items) * 16;
  const int grid = units < num_sms ? static_cast<int>(units) : num_sms;
  return launch_pdl(attn_flash_kernel, dim3(grid), dim3(THREADS), SMEM, stream, nullptr, 0, *tm_qkv, a);
}

}  // namespace laya
