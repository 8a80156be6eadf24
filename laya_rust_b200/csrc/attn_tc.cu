// Ragged attention on the 5th-generation tensor cores (tcgen05 + TMEM):
// a persistent, warp-specialised flash kernel with an online softmax.
//
// Contract (laya-rust backend/cpu/mod.rs:257-314 with the masks of
// :316-328): out = softmax(q . k^T + mask) . v per (sequence, head), q and k
// already scaled; a key is visible to a query when it is a real token of
// the same sequence and, on local layers, within +-window positions.  No
// mask tensor exists: each query row derives its visible key interval
// [lo, hi) from its sequence and the window.
//
// Work: a unit is (item, head); an item is a block of at most 128 query
// rows of one sequence (one per 128 rows) with the key blocks of 128 they
// can see (1-4; blocks outside the window skipped).  Only a sequence's own
// rows are loaded, in 32-row TMA boxes.  One CTA per SM walks the units
// blockIdx.x, blockIdx.x + gridDim.x, ...; unit k of a CTA goes to slot
// k & 1, so two units are in flight per CTA and one slot's softmax overlaps
// the other slot's MMAs and loads.
//
// Roles (608 threads):
//   warp 0      TMA producer of Q (one buffer per slot) and K blocks (a
//               3-stage ring, a stage freed once its S is computed)
//   warp 1      TMA producer of V blocks (a 3-stage ring, a stage freed once
//               its P.V is done): K loads run ahead of the P.V they wait on
//   warp 2      TMEM allocation; one thread issues the MMAs:
//                 S[slot] = Q . K_j^T          (M=128, N=128, K=64)
//                 O[slot] += P_j . [V_j | 1]   (M=128, N=80,  K=128)
//               The B operand of the second is V (64 columns) followed by an
//               all-ones block, so O's column 64 accumulates the row sums of
//               P in f32 (the sums of exactly the f16 values multiplied
//               into V).  Both run in a fixed step order shared with the
//               producers (the two slots' key-block steps alternate; each S
//               is followed by the P.V of the step before it).
//   warps 3-18  softmax, four warpgroups: (slot, half) = (0,0) (0,1) (1,0)
//               (1,1).  Thread t of a warpgroup owns query row t = TMEM lane
//               t and, of each key block, the 64 keys of its half.  Per key
//               block it reads its scores from TMEM in 32-key chunks (chunks
//               no row of the warp can see are skipped; chunks every row of
//               the warp sees fully take a path without selects), takes its
//               half's maximum, exchanges it with the other half's thread of
//               the same row through shared memory (a 64-thread named
//               barrier per slot and lane quarter), writes
//               P = 2^(s log2 e - max) with the packed f16 exponential into
//               its half of the row of P (the swizzled K-major operand
//               layout, one 64-key atom per half) and rescales its columns of
//               the row's O (and the sum column) in TMEM when the maximum P
//               is taken against moved -- only when a block's maximum exceeds
//               it by more than 8 in log2 units, so P <= 256 and most blocks
//               skip the rescale.  After the unit's last block each half scales its 32
//               of the row's 64 outputs by 1 / sum and stores them.
// Shared memory: Q 2 x 16 KB, K 3 x 16 KB, V 3 x 16 KB, ones 16 KB, P 2 x 32
// KB, the CTA's first 64 work items, the max exchange (about 212 KB).
// TMEM: S 2 x 128 columns, O 2 x 80 columns (at 256 and 384; 512 allocated).
//
// Every wait is bounded (2 s by default).  On expiry the waiting thread
// records an error code and raises the CTA's abort flag; every role stops
// waiting and working (the softmax warps still pass their named barriers,
// the same number as their partners, so none is left waiting), the MMA
// thread waits (bounded) for the MMAs it issued, the CTA lingers 2 ms so
// TMA loads in flight land, and TMEM is freed.  The host reads the error
// word after the forward.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int TQ = 128;                  // query rows per item
constexpr int TK = 128;                  // keys per block
constexpr int D = 64;                    // head dim
constexpr int DO = 80;                   // O columns: 64 outputs + the sum block
constexpr int BOX = 32;                  // rows per TMA box
constexpr int NK = 3;                    // K ring stages
constexpr int NV = 3;                    // V ring stages
constexpr int CTRL_WARPS = 3;            // Q/K producer, V producer, MMA
constexpr int SOFTMAX_WARPS = 16;
constexpr int THREADS = 32 * (CTRL_WARPS + SOFTMAX_WARPS);
constexpr int TILE_BYTES = TQ * D * 2;   // 16 KB: one [128 x 64] f16 tile
constexpr int BOX_BYTES = BOX * D * 2;   // 4 KB
constexpr int P_BYTES = 2 * TILE_BYTES;  // P [128 x 128] f16: two 64-key atoms
constexpr int MAX_UNITS = 64;            // work items cached in shared memory
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + NK * TILE_BYTES;
constexpr int OFF_ONES = OFF_V + NV * TILE_BYTES;             // after every V stage (positive LBO)
constexpr int OFF_P = OFF_ONES + TILE_BYTES;
constexpr int OFF_ITEMS = OFF_P + 2 * P_BYTES;                 // int4[MAX_UNITS]
constexpr int OFF_XMAX = OFF_ITEMS + MAX_UNITS * 16;           // f32[slot][parity][half][128]
constexpr int OFF_BAR = OFF_XMAX + 2 * 2 * 2 * TQ * 4;
// barriers: q_full[2] q_empty[2] k_full[NK] k_empty[NK] v_full[NV]
// v_empty[NV] s_full[2] p_full[2] pv_done[2] drain stuck, then the TMEM
// address and the abort flag
constexpr int NBARS = 2 + 2 + 2 * NK + 2 * NV + 2 + 2 + 2 + 2;
constexpr size_t SMEM = 1024 + OFF_BAR + NBARS * 8 + 16;
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0;                 // S[slot] at slot * 128
constexpr int O_COL = 256;               // O[slot] at 256 + slot * 128 (80 used)
constexpr float L2E = 1.4426950408889634f;
// 8 in log2 units: the most a row's scores may exceed the maximum its P is
// taken against before O is rescaled (P <= 256)
constexpr float kRescaleSlack = 8.0f / L2E;

// S: A = Q (K-major), B = K block (K-major), M = 128, N = 128
constexpr uint32_t IDESC_QK = umma_idesc_f16(TQ, TK);
// O: A = P (K-major over keys), B = [V | ones] (MN-major), M = 128, N = 80
constexpr uint32_t IDESC_PV = umma_idesc_f16(TQ, DO) | (1u << 16);

// Descriptor of an MN-major operand written with 128-byte swizzle: rows are
// K (keys), 128 B of N (64 f16) per row, 8-row groups 1024 B apart (stride
// byte offset); the next 64 N columns start `lbo` bytes further (leading
// byte offset): here the all-ones block.
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

// 2^x with the hardware approximation (relative error ~2^-22): one MUFU op.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (2^x0, 2^x1) as packed f16 (x0 in the low half): the arguments are
// rounded to f16 and one MUFU op exponentiates both.
__device__ __forceinline__ uint32_t exp2_h2(float x0, float x1) {
  uint32_t h, r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(h));
  return r;
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

// One 32-bit column of 32 lanes (the row sum).
__device__ __forceinline__ uint32_t tmem_ld_32x32b_x1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}
__device__ __forceinline__ void tmem_st_32x32b_x1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Barrier `id` (1..8) over the `count` threads of two warps.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Bits j of a 32-key chunk with a <= j < b (a, b relative to the chunk, any
// integers): the keys of the chunk one query row can see.
__device__ __forceinline__ uint32_t chunk_mask(int a, int b) {
  const int lo = a < 0 ? 0 : (a > 32 ? 32 : a);
  const int hi = b < 0 ? 0 : (b > 32 ? 32 : b);
  if (hi <= lo) return 0u;
  const uint64_t m = ((1ull << hi) - 1ull) & ~((1ull << lo) - 1ull);
  return static_cast<uint32_t>(m);
}

// A unit's item: query rows [q_row0, q_row0 + q_rows) of the sequence
// [seq0, seq1), and the key blocks [k_row0 + 128 j, ...), j < nkb, they can
// see (windowed on local layers).
struct ItemGeom {
  int q_row0, q_rows, k_row0, nkb, seq1;
};

__device__ __forceinline__ ItemGeom item_geom(const int4 it, int window) {
  // it = (first query row, query rows, sequence start row, sequence length)
  const int q0 = it.x - it.z, len = it.w;
  int lo = 0, hi = len;
  if (window >= 0) {
    lo = q0 - window > 0 ? q0 - window : 0;
    hi = q0 + it.y + window < len ? q0 + it.y + window : len;
  }
  const int kb0 = lo / TK, kb1 = (hi + TK - 1) / TK;
  return ItemGeom{it.x, it.y, it.z + kb0 * TK, kb1 - kb0 > 0 ? kb1 - kb0 : 1, it.z + len};
}

// 32-row boxes a tile of rows [r0, min(r0 + 128, end)) needs (at least one).
__device__ __forceinline__ int boxes(int r0, int end) {
  const int n = end - r0 < TQ ? end - r0 : TQ;
  return n <= 0 ? 1 : (n + BOX - 1) / BOX;
}

// The work item of this CTA's unit k (from the shared-memory cache when it
// holds it).
__device__ __forceinline__ int4 unit_item(const AttnArgs& a, const int4* cache, int k) {
  if (k < MAX_UNITS) return cache[k];
  return __ldg(a.items + ((blockIdx.x + k * gridDim.x) >> 4));
}

// The fixed order of key-block steps shared by the producers and the MMA
// thread: the two slots' steps alternate (a slot whose units are exhausted
// drops out).  Slot s holds this CTA's units k = s, s + 2, ...
struct StepIter {
  int units;
  int k0, k1, j0, j1, nkb0, nkb1, n0, n1;
  int turn;
  __device__ __forceinline__ void init(const AttnArgs& a, const int4* cache, int cta_units) {
    units = cta_units;
    k0 = 0; k1 = 1; j0 = j1 = 0; n0 = n1 = 0; turn = 0;
    nkb0 = k0 < units ? item_geom(unit_item(a, cache, k0), a.window).nkb : 1;
    nkb1 = k1 < units ? item_geom(unit_item(a, cache, k1), a.window).nkb : 1;
  }
  // Next step: slot, unit index k within the CTA, block j, its unit's block
  // count and the slot's running step count c.  False when both are done.
  __device__ __forceinline__ bool next(const AttnArgs& a, const int4* cache, int& slot, int& kk, int& jj,
                                       int& nb, int& c) {
    int s = turn;
    if ((s == 0 ? k0 : k1) >= units) s ^= 1;
    if ((s == 0 ? k0 : k1) >= units) return false;
    slot = s;
    turn = s ^ 1;
    if (s == 0) {
      kk = k0; jj = j0; nb = nkb0; c = n0++;
      if (++j0 == nkb0) {
        j0 = 0;
        k0 += 2;
        if (k0 < units) nkb0 = item_geom(unit_item(a, cache, k0), a.window).nkb;
      }
    } else {
      kk = k1; jj = j1; nb = nkb1; c = n1++;
      if (++j1 == nkb1) {
        j1 = 0;
        k1 += 2;
        if (k1 < units) nkb1 = item_geom(unit_item(a, cache, k1), a.window).nkb;
      }
    }
    return true;
  }
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const AttnArgs& a, int code,
                                         volatile int* abort_flag) {
  return mbar_wait_bounded(bar, parity, a.err, code, abort_flag, a.wait_limit_ns);
}

// Lane 0 waits (bounded) and the warp agrees on the outcome; a warp that
// already failed does not wait again.
__device__ __forceinline__ bool warp_wait(bool ok, uint64_t* bar, uint32_t parity, const AttnArgs& a,
                                          volatile int* abort_flag) {
  int w = ok ? 1 : 0;
  if (ok && (threadIdx.x & 31) == 0) w = wait_bar(bar, parity, a, kErrAttnWait, abort_flag);
  return __shfl_sync(0xffffffffu, w, 0) != 0;
}

__global__ void __launch_bounds__(THREADS, 1)
    attn_flash_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  int4* uitems = reinterpret_cast<int4*>(smem + OFF_ITEMS);
  float* xmax = reinterpret_cast<float*>(smem + OFF_XMAX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 2;
  uint64_t* k_full = q_empty + 2;
  uint64_t* k_empty = k_full + NK;
  uint64_t* v_full = k_empty + NK;
  uint64_t* v_empty = v_full + NV;
  uint64_t* s_full = v_empty + NV;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* drain = pv_done + 2;
  uint64_t* stuck_bar = drain + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stuck_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total_units = a.num_items * 16;
  const int my_units =
      static_cast<int>(blockIdx.x) < total_units ? (total_units - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);  // the eight softmax warps of the slot
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < NK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(stuck_bar, 1);  // nothing ever arrives on it (the timeout test)
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
  }
  // V rows past a sequence's end are never loaded: the V stages start as
  // zeros (then only ever hold real, finite rows), so P = 0 times a stale row
  // stays 0; the ones block feeds the row-sum columns of O
  {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    const uint4 one = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);  // f16 1.0
    for (int i = tid; i < (NV + 1) * TILE_BYTES / 16; i += THREADS)
      reinterpret_cast<uint4*>(smem + OFF_V)[i] = i < NV * TILE_BYTES / 16 ? z : one;
  }
  // the work items come from the plan upload, which precedes every kernel of
  // the forward, so they may be read before the previous kernel completes
  if (tid >= 96 && tid - 96 < MAX_UNITS && tid - 96 < my_units)
    uitems[tid - 96] = __ldg(a.items + ((blockIdx.x + (tid - 96) * gridDim.x) >> 4));
  if (warp == 2) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the zeros and ones, before the tensor core reads them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  grid_dep_wait();
  grid_dep_trigger();

  if (warp <= 1) {
    // ---- TMA producers: warp 0 Q and K, warp 1 V, both in the step order ------------
    if (lane == 0) {
      bool ok = true;
      if (a.stuck) ok = wait_bar(stuck_bar, 0, a, kErrAttnWait, abort_flag);
      const uint64_t pol = l2_evict_first();  // q/k/v are read by this launch only
      StepIter it;
      it.init(a, uitems, my_units);
      uint32_t qe_phase0 = 0, qe_phase1 = 0, e_phase = 0;
      int nq0 = 0, nq1 = 0, stage = 0;
      const int nst = warp == 0 ? NK : NV;
      int slot, kk, jj, nb, c;
      while (ok && it.next(a, uitems, slot, kk, jj, nb, c)) {
        const int h = (static_cast<int>(blockIdx.x) + kk * static_cast<int>(gridDim.x)) & 15;
        const ItemGeom g = item_geom(unit_item(a, uitems, kk), a.window);
        const int krow = g.k_row0 + jj * TK;
        const int kb = boxes(krow, g.seq1);
        if (warp == 0) {
          if (jj == 0) {
            if ((slot == 0 ? nq0 : nq1) > 0) {
              uint32_t& ph = slot == 0 ? qe_phase0 : qe_phase1;
              if (!(ok = wait_bar(&q_empty[slot], ph, a, kErrAttnWait, abort_flag))) break;
              ph ^= 1u;
            }
            if (slot == 0) ++nq0; else ++nq1;
            const int qb = boxes(g.q_row0, g.q_row0 + g.q_rows);
            mbar_arrive_expect_tx(&q_full[slot], qb * BOX_BYTES);
            for (int b = 0; b < qb; ++b)
              tma_load_2d_hint(smem + OFF_Q + slot * TILE_BYTES + b * BOX_BYTES, &tm_qkv, h * D, g.q_row0 + b * BOX,
                               &q_full[slot], pol);
          }
          if (!(ok = wait_bar(&k_empty[stage], e_phase ^ 1u, a, kErrAttnWait, abort_flag))) break;
          mbar_arrive_expect_tx(&k_full[stage], kb * BOX_BYTES);
          for (int b = 0; b < kb; ++b)
            tma_load_2d_hint(smem + OFF_K + stage * TILE_BYTES + b * BOX_BYTES, &tm_qkv, 1024 + h * D,
                             krow + b * BOX, &k_full[stage], pol);
        } else {
          if (!(ok = wait_bar(&v_empty[stage], e_phase ^ 1u, a, kErrAttnWait, abort_flag))) break;
          mbar_arrive_expect_tx(&v_full[stage], kb * BOX_BYTES);
          for (int b = 0; b < kb; ++b)
            tma_load_2d_hint(smem + OFF_V + stage * TILE_BYTES + b * BOX_BYTES, &tm_qkv, 2048 + h * D,
                             krow + b * BOX, &v_full[stage], pol);
        }
        if (++stage == nst) {
          stage = 0;
          e_phase ^= 1u;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 2) {
    // ---- MMA issuer ----------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      StepIter it;
      it.init(a, uitems, my_units);
      uint32_t qf_phase0 = 0, qf_phase1 = 0, kf_phase = 0, vf_phase = 0, pf_phase0 = 0, pf_phase1 = 0;
      int p_seen0 = 0, p_seen1 = 0;  // p_full completions consumed per slot
      int kst = 0, vst = 0;
      // descriptors: per-step operands are fixed offsets from these
      const uint32_t ones = smem_u32(smem + OFF_ONES);
      const uint64_t dq0 = umma_desc_sw128(smem_u32(smem + OFF_Q));
      const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + OFF_K));
      const uint64_t dp0 = umma_desc_sw128(smem_u32(smem + OFF_P));
      // the step issued last, whose P.V follows the next S
      bool pend = false, pend_first = false;
      int pend_slot = 0, pend_c = 0;
      // waits until slot s's p_full has completed `count` times
      auto wait_p = [&](int s, int count) {
        int& seen = s == 0 ? p_seen0 : p_seen1;
        uint32_t& ph = s == 0 ? pf_phase0 : pf_phase1;
        while (ok && seen < count) {
          ok = wait_bar(&p_full[s], ph, a, kErrAttnWait, abort_flag);
          ph ^= 1u;
          ++seen;
        }
        return ok;
      };
      auto issue_pv = [&]() {
        // P_j of the pending step is written (and its O rescaled) once p_full
        // completes for the slot's (c + 1)-th time
        if (!wait_p(pend_slot, pend_c + 1)) return;
        if (!(ok = wait_bar(&v_full[vst], vf_phase, a, kErrAttnWait, abort_flag))) return;
        tc_fence_after();
        const uint32_t va = smem_u32(smem + OFF_V + vst * TILE_BYTES);
        const uint64_t dv = desc_mn_sw128(va, ones - va);
        const uint64_t dp = dp0 + static_cast<uint64_t>(pend_slot * (P_BYTES >> 4));
        const uint32_t d = tmem + O_COL + pend_slot * 128;
#pragma unroll
        for (int kk2 = 0; kk2 < TK / 16; ++kk2)
          umma_f16(d, dp + static_cast<uint64_t>((kk2 >> 2) * (TILE_BYTES >> 4) + (kk2 & 3) * 2),
                   dv + static_cast<uint64_t>(kk2 * (2048 >> 4)), IDESC_PV, (!pend_first || kk2 > 0) ? 1u : 0u);
        umma_commit(&v_empty[vst]);
        umma_commit(&pv_done[pend_slot]);
        if (++vst == NV) {
          vst = 0;
          vf_phase ^= 1u;
        }
        pend = false;
      };
      int slot, kk, jj, nb, c;
      while (ok && it.next(a, uitems, slot, kk, jj, nb, c)) {
        // S[slot] is free once the slot's previous step has its P written
        if (!wait_p(slot, c)) break;
        if (jj == 0) {
          uint32_t& ph = slot == 0 ? qf_phase0 : qf_phase1;
          if (!(ok = wait_bar(&q_full[slot], ph, a, kErrAttnWait, abort_flag))) break;
          ph ^= 1u;
        }
        if (!(ok = wait_bar(&k_full[kst], kf_phase, a, kErrAttnWait, abort_flag))) break;
        tc_fence_after();
        const uint64_t dq = dq0 + static_cast<uint64_t>(slot * (TILE_BYTES >> 4));
        const uint64_t dk = dk0 + static_cast<uint64_t>(kst * (TILE_BYTES >> 4));
#pragma unroll
        for (int k4 = 0; k4 < D / 16; ++k4)
          umma_f16(tmem + S_COL + slot * TK, dq + static_cast<uint64_t>(2 * k4), dk + static_cast<uint64_t>(2 * k4),
                   IDESC_QK, k4 > 0 ? 1u : 0u);
        umma_commit(&s_full[slot]);
        umma_commit(&k_empty[kst]);
        if (jj == nb - 1) umma_commit(&q_empty[slot]);
        if (++kst == NK) {
          kst = 0;
          kf_phase ^= 1u;
        }
        if (pend) {
          issue_pv();
          if (!ok) break;
        }
        pend = true;
        pend_slot = slot;
        pend_c = c;
        pend_first = jj == 0;
      }
      if (ok && pend) issue_pv();
      if (!ok) *abort_flag = 1;
      // every MMA issued here completes before TMEM is released
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, a.err, kErrAttnWait, nullptr, 0);
    }
  } else {
    // ---- softmax warpgroups --------------------------------------------------------
    const int wg = (warp - CTRL_WARPS) >> 2;
    const int slot = wg >> 1, half = wg & 1;
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    const int row = q * 32 + lane;              // query row within the item
    const int bar_id = 1 + slot * 4 + q;        // this row quarter's two warps
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t t_s = t_lane + S_COL + slot * TK + half * 64;  // this half's 64 keys
    const uint32_t t_o = t_lane + O_COL + slot * 128 + half * 32;  // this half's 32 columns of O
    const uint32_t t_sum = t_lane + O_COL + slot * 128 + D;       // the row-sum column
    uint8_t* prow = smem + OFF_P + slot * P_BYTES + half * TILE_BYTES + row * 128;
    float* xmax_s = xmax + slot * (2 * 2 * TQ);
    uint32_t sf_phase = 0, pv_phase = 0;
    int par = 0;
    bool ok = true;
    for (int kk = slot; kk < my_units; kk += 2) {
      const int h = (static_cast<int>(blockIdx.x) + kk * static_cast<int>(gridDim.x)) & 15;
      const int4 it = unit_item(a, uitems, kk);
      const ItemGeom g = item_geom(it, a.window);
      const bool valid = row < g.q_rows;
      const int r_abs = g.q_row0 + row;
      int lo = 0, hi = 0;  // visible keys, absolute rows
      if (valid) {
        lo = it.z;
        hi = g.seq1;
        if (a.window >= 0) {
          lo = r_abs - a.window > lo ? r_abs - a.window : lo;
          hi = r_abs + a.window + 1 < hi ? r_abs + a.window + 1 : hi;
        }
      }
      float m_run = -INFINITY;
      for (int jj = 0; jj < g.nkb; ++jj) {
        ok = warp_wait(ok, &s_full[slot], sf_phase, a, abort_flag);
        sf_phase ^= 1u;
        if (ok) tc_fence_after();
        // keys [a0, b0) of this half's 64 are visible to the row
        const int kbase = g.k_row0 + jj * TK + half * 64;
        const int a0 = lo - kbase, b0 = hi - kbase;
        const uint32_t mask0 = chunk_mask(a0, b0), mask1 = chunk_mask(a0 - 32, b0 - 32);
        const bool any0 = __any_sync(0xffffffffu, mask0 != 0u), any1 = __any_sync(0xffffffffu, mask1 != 0u);
        const bool all0 = __all_sync(0xffffffffu, mask0 == 0xffffffffu);
        const bool all1 = __all_sync(0xffffffffu, mask1 == 0xffffffffu);
        // pass 1: this half's maximum
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          const uint32_t mask = ch ? mask1 : mask0;
          if (!ok || !(ch ? any1 : any0)) continue;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_s + 32 * ch, v);
          tmem_ld_wait();
          if (ch ? all1 : all0) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) mx[(j >> 1) & 3] = fmax3f(mx[(j >> 1) & 3], u2f(v[j]), u2f(v[j + 1]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; j += 2)
              mx[(j >> 1) & 3] = fmax3f(mx[(j >> 1) & 3], (mask >> j) & 1u ? u2f(v[j]) : -INFINITY,
                                        (mask >> (j + 1)) & 1u ? u2f(v[j + 1]) : -INFINITY);
          }
        }
        const float mh = fmax3f(mx[0], mx[1], fmaxf(mx[2], mx[3]));
        // the row's block maximum: this half's and the other half's
        xmax_s[(par * 2 + half) * TQ + row] = mh;
        named_sync(bar_id, 64);
        const float mo = xmax_s[(par * 2 + (half ^ 1)) * TQ + row];
        par ^= 1;
        // The maximum P is taken against moves only when the block's
        // maximum exceeds it by more than kRescaleSlack: P = 2^((s - m) log2 e)
        // then stays at most 2^8 (f16 holds it to the same relative
        // precision), and O and its row sum, accumulated against the same m,
        // give the same quotient -- so most blocks need no rescale of O.
        const float m_blk = fmaxf(mh, mo);
        const float m_new = (m_run == -INFINITY || m_blk > m_run + kRescaleSlack) ? fmaxf(m_run, m_blk) : m_run;
        const float m_use = m_new == -INFINITY ? 0.0f : m_new;
        const float ms = m_use * L2E;
        // O (sums included) was accumulated against m_run: rescale by
        // 2^((m_run - m_new) log2 e) when m moved; while m_run is -inf every
        // earlier P of the row was 0, so O is 0 and needs none
        const float alpha =
            (m_new == m_run || m_run == -INFINITY) ? 1.0f : fast_exp2((m_run - m_use) * L2E);
        // the slot's previous P.V must be done: P is rewritten and O rescaled
        if (jj > 0) {
          ok = warp_wait(ok, &pv_done[slot], pv_phase, a, abort_flag);
          pv_phase ^= 1u;
          if (ok) tc_fence_after();
        }
        // pass 2: P = 2^(s log2e - max) (0 where hidden) as f16 into this
        // half's atom of the row (chunk ch -> 16-byte chunks 4 ch .. 4 ch + 3)
        if (ok) {
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            const uint32_t mask = ch ? mask1 : mask0;
            uint32_t w[16];
            if (!(ch ? any1 : any0)) {
#pragma unroll
              for (int j = 0; j < 16; ++j) w[j] = 0u;
            } else {
              uint32_t v[32];
              tmem_ld_32x32b_x32(t_s + 32 * ch, v);
              tmem_ld_wait();
              if (ch ? all1 : all0) {
                // s log2 e - max for two keys per packed step
                const uint64_t l2e2 = f2_splat(L2E), nms2 = f2_splat(-ms);
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                  float a0, a1;
                  f2_get(f2_fma(f2(u2f(v[j]), u2f(v[j + 1])), l2e2, nms2), a0, a1);
                  w[j / 2] = exp2_h2(a0, a1);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                  w[j / 2] = exp2_h2((mask >> j) & 1u ? fmaf(u2f(v[j]), L2E, -ms) : -INFINITY,
                                     (mask >> (j + 1)) & 1u ? fmaf(u2f(v[j + 1]), L2E, -ms) : -INFINITY);
              }
            }
#pragma unroll
            for (int x = 0; x < 4; ++x)
              *reinterpret_cast<uint4*>(prow + (((4 * ch + x) ^ (row & 7)) << 4)) =
                  make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
          }
        }
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows' maximum grew (alpha is 1 elsewhere);
        // half 1 also rescales the row-sum column
        if (ok && jj > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o, o);
          uint32_t sv = 0;
          if (half) sv = tmem_ld_32x32b_x1(t_sum);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(u2f(o[j]) * alpha);
          tmem_st_32x32b_x32(t_o, o);
          if (half) tmem_st_32x32b_x1(t_sum, __float_as_uint(u2f(sv) * alpha));
          tmem_st_wait();
        }
        m_run = m_new;
        fence_proxy_async_smem();  // P (generic writes) visible to the tensor core
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&p_full[slot]);
      }
      // the unit's last P.V, then the epilogue: each half scales its 32 of
      // the row's 64 values by 1 / (row sum) and stages them as f16 in the
      // slot's P buffer (free now: its last P.V is done), row r at r * 128
      // bytes, 16-byte chunk c at (c ^ (r & 7)); then the row quarter's two
      // warps store their 32 rows with whole 128-byte lines per row
      ok = warp_wait(ok, &pv_done[slot], pv_phase, a, abort_flag);
      pv_phase ^= 1u;
      uint8_t* stage = smem + OFF_P + slot * P_BYTES;
      if (ok) {
        tc_fence_after();
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o, o);
        const uint32_t sv = tmem_ld_32x32b_x1(t_sum);
        tmem_ld_wait();
        const float l = u2f(sv);
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
        for (int x = 0; x < 4; ++x)
          *reinterpret_cast<uint4*>(stage + row * 128 + (((4 * half + x) ^ (row & 7)) << 4)) =
              make_uint4(pack_half2(u2f(o[8 * x]) * inv, u2f(o[8 * x + 1]) * inv),
                         pack_half2(u2f(o[8 * x + 2]) * inv, u2f(o[8 * x + 3]) * inv),
                         pack_half2(u2f(o[8 * x + 4]) * inv, u2f(o[8 * x + 5]) * inv),
                         pack_half2(u2f(o[8 * x + 6]) * inv, u2f(o[8 * x + 7]) * inv));
      }
      named_sync(bar_id, 64);
      if (ok) {
        // 32 rows x 8 chunks of this quarter; thread i of the pair takes
        // chunks i, i + 64, i + 128, i + 192 (8 consecutive threads per row)
        const int i = half * 32 + lane;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int cidx = i + 64 * x;
          const int rr = q * 32 + (cidx >> 3), c = cidx & 7;
          if (rr < g.q_rows) {
            const uint4 vv = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
            *reinterpret_cast<uint4*>(a.out + static_cast<size_t>(g.q_row0 + rr) * 1024 + h * D + c * 8) = vv;
          }
        }
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
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_attention_tc(const CUtensorMap* tm_qkv, const AttnArgs& a, int num_sms, cudaStream_t stream) {
  if (a.num_items <= 0) return cudaSuccess;
  if (!a.items || !a.out || !a.err || num_sms <= 0) return cudaErrorInvalidValue;
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
