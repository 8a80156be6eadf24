// Ragged attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as attention.cu (laya-rust backend/cpu/mod.rs:257-328:
// softmax(q.k^T + mask) v with q, k pre-scaled; a key is visible when it is
// a real token of the sequence and, on local layers, within +-64 positions),
// computed per (128-query block, head) CTA:
//
//   TMA      Q [128 x 64], K and V blocks [128 keys x 64] of one head, read
//            straight out of the token-major qkv buffer, 128-byte swizzle
//   MMA 1    S = Q . K^T  -> TMEM columns [0, 128)      (M=128, N=128, K=64)
//   softmax  thread t owns query row t = TMEM lane t: it reads its 128
//            scores, masks, exponentiates and writes its row of P (f16) to
//            shared memory in the K-major swizzled operand layout
//   MMA 2    O += P . V -> TMEM columns [128, 192)        (M=128, N=64, K=128)
//            V is consumed as an MN-major operand (d contiguous)
//   store    thread t scales its O row by 1 / rowsum and writes 64 f16
//
// When the visible keys span more than one 128-key block (sequences longer
// than 128, or the +-64 band of a 128-row block), the softmax is exact in two
// passes: pass 1 runs MMA 1 over every key block to get each row's maximum
// and sum; pass 2 recomputes S block by block, writes P = exp(s - max) and
// accumulates O.  No rescaling of O is needed.  Key blocks outside the band
// are skipped.
//
// Sequences of at most 128 tokens take the single-pass variant, with whole
// consecutive sequences packed into one 128-row tile (they are adjacent in
// the compacted rows): each query row's visible keys are the interval of its
// own sequence (+-64 on local layers), so the packing changes no result and
// the tiles carry fewer padding rows.  48 KB shared memory and 128 TMEM
// columns (P aliases Q and K, O aliases S): four CTAs per SM.  Longer
// sequences: one CTA per (128-row block, head), 82 KB shared memory and 256
// TMEM columns, two CTAs per SM.  Every wait is bounded.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int TQ = 128;
constexpr int TK = 128;
constexpr int D = 64;
constexpr int THREADS = 128;
constexpr int TILE_BYTES = TQ * D * 2;  // 16 KB: one [128 x 64] f16 tile
constexpr int P_BYTES = 2 * TILE_BYTES; // P: two 64-key K atoms
// Two layouts.  Sequences of at most 128 tokens need one key block: P
// overwrites the Q and K tiles once S is computed and O overwrites S in TMEM,
// so a CTA needs 48 KB and 128 TMEM columns (four CTAs per SM).  Longer
// sequences keep Q, K, V, P and separate S / O columns (two CTAs per SM).
template <bool kSingle>
struct Layout {
  static constexpr int TMEM_COLS = kSingle ? 128 : 256;
  static constexpr int S_COL = 0;
  static constexpr int O_COL = kSingle ? 0 : 128;
  static constexpr int P_OFF = kSingle ? 0 : 3 * TILE_BYTES;
  static constexpr size_t SMEM = 1024 + 3 * TILE_BYTES + (kSingle ? 0 : P_BYTES) + 128;
  static constexpr size_t BAR_OFF = 3 * TILE_BYTES + (kSingle ? 0 : P_BYTES);
  static constexpr int MIN_BLOCKS = kSingle ? 4 : 2;
};
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

// Keys visible to one query row r: [lo, hi) (the row's +-window band within
// the sequence, or the whole sequence).  A 32-key chunk starting at j0 is
// wholly visible, wholly hidden, or straddles an edge.
struct RowRange {
  int lo, hi;
  __device__ __forceinline__ bool full(int j0) const { return j0 >= lo && j0 + 32 <= hi; }
  __device__ __forceinline__ bool none(int j0) const { return j0 + 32 <= lo || j0 >= hi; }
  __device__ __forceinline__ float mask(float s, int j) const { return (j >= lo && j < hi) ? s : -INFINITY; }
};

// Maximum of the visible scores of one 32-key chunk.
__device__ __forceinline__ float chunk_max(const uint32_t (&v)[32], const RowRange& rr, int j0) {
  float mx = -INFINITY;
  if (rr.none(j0)) return mx;
  if (rr.full(j0)) {
#pragma unroll
    for (int j = 0; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(v[j]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) mx = fmaxf(mx, rr.mask(__uint_as_float(v[j]), j0 + j));
  }
  return mx;
}

struct Ctl {
  uint64_t* kv_bar;
  uint64_t* s_bar;
  uint64_t* o_bar;
  int* err;
  uint32_t kv_phase, s_phase, o_phase;
};

// Every thread observes the barrier itself (bounded); the warp agrees on the
// outcome.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t& phase, int* err, int code) {
  const bool mine = mbar_wait_bounded(bar, phase, err, code, nullptr);
  phase ^= 1u;
  return __all_sync(0xffffffffu, mine) != 0;
}

template <bool kSingle>
__global__ void __launch_bounds__(THREADS, Layout<kSingle>::MIN_BLOCKS)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnArgs a, int* err) {
  using Lay = Layout<kSingle>;
  constexpr int TMEM_COLS = Lay::TMEM_COLS, S_COL = Lay::S_COL, O_COL = Lay::O_COL;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + TILE_BYTES;
  uint8_t* sV = smem + 2 * TILE_BYTES;
  uint8_t* sP = smem + Lay::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::BAR_OFF);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3);

  grid_dep_wait();
  grid_dep_trigger();
  const int tid = threadIdx.x, warp = tid >> 5;
  const int2 blk = a.blocks[blockIdx.x];
  const int h = blockIdx.y;
  // kSingle: blk = (first row, rows) of a tile of whole sequences packed back
  // to back; `len` is then the tile's row count and positions count from its
  // first row.  Otherwise blk = (sequence, first query row).
  const int b = kSingle ? 0 : blk.x, q0 = kSingle ? 0 : blk.y;
  const int len = kSingle ? blk.y : a.seq_len[b];
  const int row_base = kSingle ? blk.x : a.seq_start[b];
  const int window = a.window;

  int k_lo = 0, k_hi = len;
  if (window >= 0) {
    k_lo = q0 - window;
    if (k_lo < 0) k_lo = 0;
    const int q_last = (q0 + TQ < len ? q0 + TQ : len) - 1;
    k_hi = q_last + window + 1;
    if (k_hi > len) k_hi = len;
  }
  const int kb0 = k_lo / TK, kb1 = (k_hi + TK - 1) / TK;
  // the host routes sequences of at most 128 tokens (one key block for every
  // row, global or windowed) to kSingle launches and the rest to the others
  constexpr bool single = kSingle;

  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
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
  Ctl c{&bars[0], &bars[1], &bars[2], err, 0, 0, 0};

  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int r = q0 + tid;  // this thread's query position
  const int xq = h * D, xk = 1024 + h * D, xv = 2048 + h * D;

  // q/k/v tiles are read by this layer's attention only: evict-first
  const uint64_t pol = l2_evict_first();
  auto load_kv = [&](int kb, bool with_q, bool with_v) {
    if (tid == 0) {
      mbar_arrive_expect_tx(c.kv_bar, TILE_BYTES * (1 + (with_q ? 1 : 0) + (with_v ? 1 : 0)));
      if (with_q) tma_load_2d_hint(sQ, &tm_qkv, xq, row_base + q0, c.kv_bar, pol);
      tma_load_2d_hint(sK, &tm_qkv, xk, row_base + kb * TK, c.kv_bar, pol);
      if (with_v) tma_load_2d_hint(sV, &tm_qkv, xv, row_base + kb * TK, c.kv_bar, pol);
    }
  };
  auto mma_s = [&]() {
    if (tid == 0) {
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
      for (int k = 0; k < D / 16; ++k)
        umma_f16(tmem + S_COL, umma_desc_sw128(qa + k * 32), umma_desc_sw128(ka + k * 32), IDESC_QK, k > 0);
      umma_commit(c.s_bar);
    }
  };

  bool ok = true;
  float m_row = -INFINITY, l_row = 0.0f;
  RowRange rr{0, len};
  if (kSingle) {
    // the keys of this row's own sequence (tile-relative), +-window on
    // local layers
    rr.lo = rr.hi = 0;
    if (r < len) {
      const int s = a.rowseq[row_base + r];
      const int st = a.seq_start[s] - row_base, en = st + a.seq_len[s];
      rr.lo = window >= 0 && r - window > st ? r - window : st;
      rr.hi = window >= 0 && r + window + 1 < en ? r + window + 1 : en;
    }
  } else {
    if (window >= 0) {
      rr.lo = r - window > 0 ? r - window : 0;
      rr.hi = r + window + 1 < len ? r + window + 1 : len;
    }
    if (r >= len) rr.hi = rr.lo;  // a row past the sequence: never stored, no scores
  }

  // This row of S is streamed from TMEM one 32-key chunk at a time (a
  // second read is cheaper than holding 128 scores in registers).
  auto load_s = [&]() { tc_fence_after(); };
  auto block_max = [&](int kb) {
    float mx = -INFINITY;
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_lane + S_COL + 32 * i, v);
      tmem_ld_wait();
      mx = fmaxf(mx, chunk_max(v, rr, kb * TK + 32 * i));
    }
    return mx;
  };
  // sum over visible keys of 2^(s*log2e - ms); with `write_p`, the f16
  // values go to this row of P (chunk i -> K atom i/2, 16-byte chunks 4*(i%2)..)
  auto block_exp = [&](int kb, float ms, bool write_p) {
    float sum = 0.0f;
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int j0 = kb * TK + 32 * i;
      uint32_t sv[32];
      tmem_ld_32x32b_x32(t_lane + S_COL + 32 * i, sv);
      tmem_ld_wait();
      uint32_t w[16];
      if (rr.none(j0)) {
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = 0u;
      } else if (rr.full(j0)) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = fast_exp2(fmaf(u2f(sv[j]), L2E, -ms));
          const float p1 = fast_exp2(fmaf(u2f(sv[j + 1]), L2E, -ms));
          sum += p0 + p1;
          w[j / 2] = pack_half2(p0, p1);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = fast_exp2(fmaf(rr.mask(u2f(sv[j]), j0 + j), L2E, -ms));
          const float p1 = fast_exp2(fmaf(rr.mask(u2f(sv[j + 1]), j0 + j + 1), L2E, -ms));
          sum += p0 + p1;
          w[j / 2] = pack_half2(p0, p1);
        }
      }
      if (write_p) {
        uint8_t* prow = sP + (i >> 1) * TILE_BYTES + tid * 128;
        const int ch0 = (i & 1) * 4;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(prow + (((ch0 + q) ^ (tid & 7)) << 4)) =
              make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      }
    }
    return sum;
  };

  // pass 1 (several key blocks): row maximum and sum of exp over all blocks
  if (!single) {
    for (int kb = kb0; kb < kb1 && ok; ++kb) {
      load_kv(kb, kb == kb0, false);
      ok = wait_all(c.kv_bar, c.kv_phase, err, kErrAttnWait);
      if (!ok) break;
      mma_s();
      ok = wait_all(c.s_bar, c.s_phase, err, kErrAttnWait);
      if (!ok) break;
      load_s();
      const float m_new = fmaxf(m_row, block_max(kb));
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      const float sum = block_exp(kb, m_use * L2E, false);
      l_row = l_row * fast_exp2((m_row - m_use) * L2E) + sum;
      m_row = m_new;
      tc_fence_before();
      __syncthreads();  // S read by all before the next MMA overwrites it
    }
  }

  // pass 2 (or the only pass): P = exp(s - max) per block, O += P . V
  for (int kb = kb0; kb < kb1 && ok; ++kb) {
    load_kv(kb, single && kb == kb0, true);
    ok = wait_all(c.kv_bar, c.kv_phase, err, kErrAttnWait);
    if (!ok) break;
    mma_s();
    ok = wait_all(c.s_bar, c.s_phase, err, kErrAttnWait);
    if (!ok) break;
    load_s();
    if (single) m_row = block_max(kb);
    const float m_use = m_row == -INFINITY ? 0.0f : m_row;
    const float sum = block_exp(kb, m_use * L2E, true);
    if (single) l_row = sum;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();  // P complete, S no longer read
    if (tid == 0) {
      tc_fence_after();
      const uint32_t pa = smem_u32(sP), va = smem_u32(sV);
#pragma unroll
      for (int kk = 0; kk < TK / 16; ++kk)
        umma_f16(tmem + O_COL, umma_desc_sw128(pa + (kk >> 2) * TILE_BYTES + (kk & 3) * 32),
                 desc_mn_sw128(va + kk * 2048), IDESC_PV, (kb > kb0 || kk > 0) ? 1u : 0u);
      umma_commit(c.o_bar);
    }
    // P, K and V are reused next block: wait until the MMAs reading them finish
    ok = wait_all(c.o_bar, c.o_phase, err, kErrAttnWait);
  }

  if (ok) {
    tc_fence_after();
    uint32_t o0[32], o1[32];
    tmem_ld_32x32b_x32(t_lane + O_COL, o0);
    tmem_ld_32x32b_x32(t_lane + O_COL + 32, o1);
    tmem_ld_wait();
    if (r < len) {
      const float inv = l_row > 0.0f ? 1.0f / l_row : 0.0f;
      uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(row_base + r) * 1024 + h * D);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dst[q] = make_uint4(pack_half2(u2f(o0[8 * q]) * inv, u2f(o0[8 * q + 1]) * inv),
                            pack_half2(u2f(o0[8 * q + 2]) * inv, u2f(o0[8 * q + 3]) * inv),
                            pack_half2(u2f(o0[8 * q + 4]) * inv, u2f(o0[8 * q + 5]) * inv),
                            pack_half2(u2f(o0[8 * q + 6]) * inv, u2f(o0[8 * q + 7]) * inv));
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dst[4 + q] = make_uint4(pack_half2(u2f(o1[8 * q]) * inv, u2f(o1[8 * q + 1]) * inv),
                                pack_half2(u2f(o1[8 * q + 2]) * inv, u2f(o1[8 * q + 3]) * inv),
                                pack_half2(u2f(o1[8 * q + 4]) * inv, u2f(o1[8 * q + 5]) * inv),
                                pack_half2(u2f(o1[8 * q + 6]) * inv, u2f(o1[8 * q + 7]) * inv));
    }
  } else if (tid == 0) {
    // a wait expired: let loads and MMAs already issued finish before teardown
    umma_commit(c.o_bar);
    mbar_wait_bounded(c.o_bar, c.o_phase, err, kErrAttnWait, nullptr);
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

template <bool kSingle>
cudaError_t launch_one(const CUtensorMap* tm_qkv, const AttnArgs& a, int num_blocks, int* err, cudaStream_t stream) {
  if (num_blocks == 0) return cudaSuccess;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  constexpr size_t smem = Layout<kSingle>::SMEM;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attn_tc_kernel<kSingle>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(attn_tc_kernel<kSingle>, dim3(num_blocks, 16), dim3(THREADS), smem, stream, nullptr, 0,
                    *tm_qkv, a, err);
}

}  // namespace

cudaError_t launch_attention_tc(const CUtensorMap* tm_qkv, const AttnArgs& a, int num_blocks, bool short_seqs,
                                int* err, cudaStream_t stream) {
  return short_seqs ? launch_one<true>(tm_qkv, a, num_blocks, err, stream)
                    : launch_one<false>(tm_qkv, a, num_blocks, err, stream);
}

}  // namespace laya
