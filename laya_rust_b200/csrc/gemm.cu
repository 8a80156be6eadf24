// Persistent 2-SM tcgen05 GEMM for sm_100a with fused epilogues.
//
//   out = epilogue(A[M,K] . W[N,K]^T)      A, W f16 K-major, f32 accumulate
//
// Replaces the reference's cuBLAS FP32 calls `mm`/`linear` (laya-rust
// src/backend/cuda/mod.rs:223-255) together with the element kernels that
// follow them: k_split_qkv (RoPE + scale, kernels.rs:135-163), k_add
// (residual, :78-82), k_gelu_mul (GeGLU, :104-112), k_add_bias/k_relu
// (:84-102).  Semantics follow the CPU op contract (backend/cpu/mod.rs:80-126,
// 202-255, 341-370).
//
// A cluster of two CTAs (two SMs) owns one 256 x BN output tile at a time and
// walks the tile list persistently.  CTA r of the pair holds A rows
// [128r, 128r+128) and W rows [r*BN/2, (r+1)*BN/2) of every k-block; the
// leader CTA (r = 0) issues tcgen05.mma.cta_group::2 (M=256, N=BN, K=16),
// which reads both CTAs' shared memory and leaves rows 128r.. of the f32
// accumulator in CTA r's TMEM.  Per CTA:
//   warp 0      TMA producer into a 6-stage ring (32 KB per stage for
//               BN=256); both CTAs' loads complete on the leader's barrier
//   warp 1      TMEM allocation (both CTAs); MMA issue (leader only);
//               accumulators double-buffered in TMEM (2 x BN columns)
//   warps 2-9   epilogue, two warps per TMEM lane quarter (one per column
//               half of the tile): tcgen05.ld of 32 lanes, fused math, a
//               128-byte-swizzled shared staging tile, then a TMA store
//               (or TMA reduce-add for the f32 residual) of 32 rows at a time
// With kEpiPartial (small M), a work unit is a (tile, K part) pair: the
// clusters split each tile's K loop and store f32 part sums, which the next
// row kernel adds in part order.  With kEpiResidTail (a residual GEMM whose
// tiles leave the last wave mostly idle), the tiles of whole waves add into
// the residual stream and the tiles of the last row blocks are split into K
// parts the same way, so the last wave is short.
// No TMA load in this kernel uses multicast; every CTA loads its own operand
// halves.  The MMA completion signal is delivered to both CTAs of the pair
// with tcgen05.commit's cluster-multicast form.
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace laya {

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LAYA_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}


namespace {

constexpr int BM = kGemmBM;            // 256 rows per cluster tile
constexpr int BK = kGemmBK;            // 64
constexpr int CTA_ROWS = BM / 2;       // 128 rows per CTA
constexpr int EPI_WARPS = 8;           // two per TMEM lane quarter, one per column half
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int STAGING_BYTES = 4096;    // 32 rows x 128 B
constexpr int BAR_BYTES = 256;
constexpr size_t SMEM_LIMIT = 232448;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = CTA_ROWS * BK * 2;        // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;        // BN=256: 16 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 6 : 8;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr size_t RING = static_cast<size_t>(STAGES) * STAGE_BYTES;
  static constexpr size_t STAGING = static_cast<size_t>(EPI_WARPS) * STAGING_BYTES;
  static constexpr size_t SMEM = 1024 + RING + STAGING + BAR_BYTES;
  static_assert(SMEM <= SMEM_LIMIT, "shared memory budget");
};

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D TMA load into this CTA's smem whose completion bytes go to the barrier
// at cluster address `bar` (the leader CTA's barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// The same with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_pair_hint(void* smem_dst, const CUtensorMap* m, int x, int y,
                                                      uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

// Reduce-add into the f32 residual stream, which is kept in L2 (evict-last).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* m, const void* smem_src, int x, int y) {
  asm volatile(
      "{\n\t.reg .b64 pol;\n\t"
      "createpolicy.fractional.L2::evict_last.b64 pol, 1.0;\n\t"
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group.L2::cache_hint"
      " [%0, {%2, %3}], [%1], pol;\n\t}" ::"l"(reinterpret_cast<uint64_t>(m)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the barrier at this smem offset in every CTA of the pair
// when all previously issued MMAs of this thread have completed.
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Arrives once on this CTA's own barrier when the MMAs have completed.
__device__ __forceinline__ void umma2_commit_own(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Writes one thread's 128-byte row (8 x 16 B) of a 32-row staging tile laid
// out the way a SWIZZLE_128B tensor map expects: 16-byte chunk j of row r at
// r*128 + ((j ^ (r & 7)) * 16).
__device__ __forceinline__ void stage_row(uint8_t* stage, int r, const uint32_t (&w)[32]) {
  uint8_t* row = stage + r * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// Per-warp epilogue state: one staging buffer, refilled once the previous
// TMA store from it has read it.  `active` is false for a 32-row slab that
// lies wholly past the last row (nothing is stored).
struct Stager {
  uint8_t* buf;
  int lane;
  bool active;
  __device__ __forceinline__ uint8_t* acquire() {
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
    return buf;
  }
  __device__ __forceinline__ void store(const CUtensorMap* m, int x, int y, bool reduce) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0 && active) {
      if (reduce) tma_reduce_add_2d(m, buf, x, y);
      else tma_store_2d(m, buf, x, y);
      bulk_commit();
    }
  }
};

// A persistent work unit: an output tile and the K range [kb0, kb1) of it
// this unit accumulates; `part` is the K part (kEpiPartial, and the split
// tail tiles of kEpiResidTail) and `tail` marks those tail units.
struct Unit {
  int tile, part, kb0, kb1;
  bool tail;
};

template <int EPI>
__device__ __forceinline__ Unit unit_of(int u, const GemmArgs& a, int num_kb) {
  Unit w{u, 0, 0, num_kb, false};
  if constexpr (EPI == kEpiPartial) {
    const int S = a.splits;
    w.tile = u / S;
    w.part = u - w.tile * S;
    w.kb0 = w.part * num_kb / S;
    w.kb1 = (w.part + 1) * num_kb / S;
  } else if constexpr (EPI == kEpiResidTail) {
    if (u >= a.main_tiles) {
      const int S = a.splits, v = u - a.main_tiles;
      w.tile = a.main_tiles + v / S;
      w.part = v - (v / S) * S;
      w.kb0 = w.part * num_kb / S;
      w.kb1 = (w.part + 1) * num_kb / S;
      w.tail = true;
    }
  }
  return w;
}

// Epilogue of one warp: 32 rows (TMEM lanes) and column half `hc` of the
// tile, i.e. columns [hc*BN/2, (hc+1)*BN/2) (for GeGLU: output columns
// [hc*BN/4, (hc+1)*BN/4), from gate and up columns of that range).
// `with_bias`: the f32 epilogues add a.bias (when set) -- once per output
// element, so only by whole tiles and by K part 0 of a split tile.
template <int EPI, int BN>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, const CUtensorMap* tmOut, Stager& st,
                                              uint32_t t_row, int row0, int row, int n0, int hc, int yoff,
                                              bool reduce, bool with_bias) {
  const bool valid = row < a.M;
  const int r = row - row0;  // row within this warp's 32-row slab
  const int cb = hc * (BN / 2), ce = cb + BN / 2;
  if constexpr (EPI == kEpiQkvRope) {
    const int part = n0 / 1024;
    if (part < 2) {
      const int p = valid ? a.pos[row] : 0;
      const float4* c4 = reinterpret_cast<const float4*>(a.cosb + p * 32);
      const float4* s4 = reinterpret_cast<const float4*>(a.sinb + p * 32);
      // (cos, sin) of the row's position for dims j, j + 1, as packed pairs
      uint64_t cs2[16], sn2[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 c = __ldg(c4 + i), s = __ldg(s4 + i);
        cs2[2 * i] = f2(c.x, c.y);
        cs2[2 * i + 1] = f2(c.z, c.w);
        sn2[2 * i] = f2(s.x, s.y);
        sn2[2 * i + 1] = f2(s.z, s.w);
      }
      const uint64_t sc2 = f2_splat(a.scale);
#pragma unroll 1
      for (int hh = cb / 64; hh < ce / 64; ++hh) {
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(t_row + hh * 64, lo);
        tmem_ld_32x32b_x32(t_row + hh * 64 + 32, hi);
        tmem_ld_wait();
        uint32_t w[32];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          // rotate-half RoPE, two dims per packed step:
          //   d < 32: (q c - q[d+32] s) scale ; d >= 32: (q c + q[d-32] s) scale
          const uint64_t A = f2(u2f(lo[j]), u2f(lo[j + 1])), B = f2(u2f(hi[j]), u2f(hi[j + 1]));
          const uint64_t C = cs2[j / 2], S = sn2[j / 2];
          float r0, r1, s0, s1;
          f2_get(f2_mul(f2_sub(f2_mul(A, C), f2_mul(B, S)), sc2), r0, r1);
          f2_get(f2_mul(f2_fma(A, S, f2_mul(B, C)), sc2), s0, s1);
          w[j / 2] = pack_half2(r0, r1);
          w[16 + j / 2] = pack_half2(s0, s1);
        }
        uint8_t* s = st.acquire();
        stage_row(s, r, w);
        st.store(tmOut, n0 + hh * 64, row0, false);
      }
    } else {
#pragma unroll 1
      for (int c0 = cb; c0 < ce; c0 += 64) {
        uint32_t v0[32], v1[32];
        tmem_ld_32x32b_x32(t_row + c0, v0);
        tmem_ld_32x32b_x32(t_row + c0 + 32, v1);
        tmem_ld_wait();
        uint32_t w[32];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          w[j / 2] = pack_half2(u2f(v0[j]), u2f(v0[j + 1]));
          w[16 + j / 2] = pack_half2(u2f(v1[j]), u2f(v1[j + 1]));
        }
        uint8_t* s = st.acquire();
        stage_row(s, r, w);
        st.store(tmOut, n0 + c0, row0, false);
      }
    }
  } else if constexpr (EPI == kEpiQkvBias || EPI == kEpiBiasRelu) {
    const float sc = (EPI == kEpiQkvBias && n0 / 1024 < 2) ? a.scale : 1.0f;
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 64) {
      uint32_t v0[32], v1[32];
      tmem_ld_32x32b_x32(t_row + c0, v0);
      tmem_ld_32x32b_x32(t_row + c0 + 32, v1);
      tmem_ld_wait();
      const float* b = a.bias + n0 + c0;
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float x0 = u2f(v0[j]) + __ldg(b + j), x1 = u2f(v0[j + 1]) + __ldg(b + j + 1);
        float y0 = u2f(v1[j]) + __ldg(b + 32 + j), y1 = u2f(v1[j + 1]) + __ldg(b + 33 + j);
        if constexpr (EPI == kEpiBiasRelu) {
          x0 = fmaxf(x0, 0.0f); x1 = fmaxf(x1, 0.0f); y0 = fmaxf(y0, 0.0f); y1 = fmaxf(y1, 0.0f);
        } else {
          x0 *= sc; x1 *= sc; y0 *= sc; y1 *= sc;
        }
        w[j / 2] = pack_half2(x0, x1);
        w[16 + j / 2] = pack_half2(y0, y1);
      }
      uint8_t* s = st.acquire();
      stage_row(s, r, w);
      st.store(tmOut, n0 + c0, row0, false);
    }
  } else if constexpr (EPI == kEpiResid || EPI == kEpiStoreF32 || EPI == kEpiPartial || EPI == kEpiResidTail) {
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      if (with_bias && a.bias) {
        const float* b = a.bias + n0 + c0;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(u2f(v[j]) + __ldg(b + j));
      }
      uint8_t* s = st.acquire();
      stage_row(s, r, v);
      // a part's rows start at yoff (K parts); 0 otherwise.  `reduce`: add
      // into the residual stream instead of storing
      st.store(tmOut, n0 + c0, row0 + yoff, reduce);
    }
  } else if constexpr (EPI == kEpiGeglu) {
    // narrow tiles (64 gate | 64 up columns): the column-half-0 warps write
    // all 64 outputs, the other four have none
    if (BN == kGemmBNNarrow && hc == 1) return;
    const int oc0 = (n0 / BN) * (BN / 2);
#pragma unroll 1
    for (int c0 = cb / 2; c0 < ce / 2; c0 += 64) {
      if (oc0 + c0 >= a.n_valid) break;
      // 16 gate and 16 up columns per TMEM load: the 64 outputs' GELU
      // chains then fit in registers and interleave
      uint32_t w[32];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t g[16], u[16];
        tmem_ld_32x32b_x16(t_row + c0 + 16 * q4, g);
        tmem_ld_32x32b_x16(t_row + BN / 2 + c0 + 16 * q4, u);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          // two columns per packed step: gelu(gate) . up
          float y0, y1;
          f2_get(f2_mul(gelu_erf2(f2(u2f(g[j]), u2f(g[j + 1]))), f2(u2f(u[j]), u2f(u[j + 1]))), y0, y1);
          w[8 * q4 + j / 2] = pack_half2(y0, y1);
        }
      }
      uint8_t* s = st.acquire();
      stage_row(s, r, w);
      st.store(tmOut, oc0 + c0, row0, false);
    }
  } else {  // kEpiScorer
    float s = 0.0f;
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      const float* b = a.bias + n0 + c0;
      const float* w = a.wvec + n0 + c0;
      // two columns per packed step; the two running sums are added at the end
      uint64_t acc2 = f2_splat(0.0f);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const uint64_t g = gelu_erf2(f2(u2f(v[j]) + __ldg(b + j), u2f(v[j + 1]) + __ldg(b + j + 1)));
        acc2 = f2_fma(g, f2(__ldg(w + j), __ldg(w + j + 1)), acc2);
      }
      float s0, s1;
      f2_get(acc2, s0, s1);
      s += s0 + s1;
    }
    if (valid) static_cast<float*>(a.out)[static_cast<size_t>(2 * (n0 / BN) + hc) * a.ldo + row] = s;
  }
}

template <int EPI, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmOut2,
                   const GemmArgs args) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* staging = smem + C::RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* stuck_bar = drain + 1;  // nothing ever arrives on it (the timeout test)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stuck_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  // tile t covers row block t / num_n and column tile t % num_n: the
  // clusters running at one time share a few A row blocks
  const int num_m = (args.M + BM - 1) / BM;
  const int num_n = args.N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = args.K / BK;
  // work units (unit_of): one per tile, or per (tile, K part) for
  // kEpiPartial and for the tail tiles of kEpiResidTail; part p of S covers
  // k-blocks [p * num_kb / S, (p + 1) * num_kb / S)
  const int num_units = EPI == kEpiPartial    ? num_tiles * args.splits
                        : EPI == kEpiResidTail ? args.main_tiles + (num_tiles - args.main_tiles) * args.splits
                                               : num_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(stuck_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_holder, C::TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barrier inits and TMEM allocation visible cluster-wide
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // the prologue above touches only shared memory, TMEM and the tensor maps
  grid_dep_wait();
  grid_dep_trigger();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if (args.stuck)
        ok = mbar_wait_bounded(stuck_bar, 0, args.err, kErrGemmProducerWait, abort_flag, args.wait_limit_ns);
      // the A operand is read by the num_n clusters working on its row block
      // at about the same time, and not after: evict-first
      const uint64_t pol_a = l2_evict_first();
      for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
        const Unit w = unit_of<EPI>(u, args, num_kb);
        const int m0 = (w.tile / num_n) * BM + static_cast<int>(rank) * CTA_ROWS;
        int n0 = (w.tile % num_n) * BN + static_cast<int>(rank) * (BN / 2);
        if constexpr (EPI == kEpiGeglu && BN == kGemmBNNarrow) {
          // a narrow GeGLU tile t pairs 64 gate rows with their 64 up rows:
          // in the co-tiled weight (256-row groups: 128 gate | 128 up) those
          // are rows 256 (t / 2) + 64 (t % 2) (CTA 0) and 128 further (CTA 1)
          const int t = w.tile % num_n;
          n0 = 256 * (t >> 1) + 128 * static_cast<int>(rank) + 64 * (t & 1);
        }
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, args.err, kErrGemmProducerWait, abort_flag,
                                 args.wait_limit_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb = map_to_rank(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          tma_load_2d_pair_hint(sA + stage * C::A_BYTES, &tmA, kb * BK, m0, fb, pol_a);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, kb * BK, n0, fb);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok || *abort_flag) {
        // give loads already in flight time to land before teardown (also
        // when another role of this CTA gave up while this loop completed)
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 2000000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
        const Unit w = unit_of<EPI>(u, args, num_kb);
        const int kb0 = w.kb0, kb1 = w.kb1;
        if (!mbar_wait_bounded(&tempty[acc], aphase ^ 1u, args.err, kErrGemmMmaWait, abort_flag, args.wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, args.err, kErrGemmMmaWait, abort_flag, args.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma2_f16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32), idesc,
                      (kb != kb0 || k != 0) ? 1u : 0u);
          umma2_commit_both(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma2_commit_both(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aphase ^= 1u;
      }
      // every MMA issued here completes before TMEM is released
      umma2_commit_own(drain);
      mbar_wait_bounded(drain, 0, args.err, kErrGemmTeardownWait, nullptr);
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int hc = ew / 4;   // column half of the tile
    Stager st{staging + ew * STAGING_BYTES, lane, true};
    const uint32_t tempty_leader[2] = {map_to_rank(smem_u32(&tempty[0]), 0), map_to_rank(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t aphase = 0;
    for (int u = cluster_id; u < num_units; u += num_clusters) {
      const Unit w = unit_of<EPI>(u, args, num_kb);
      const int tile = w.tile;
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_bounded(&tfull[acc], aphase, args.err, kErrGemmEpilogueWait, abort_flag, args.wait_limit_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int m0 = (tile / num_n) * BM + static_cast<int>(rank) * CTA_ROWS;
      const int n0 = (tile % num_n) * BN;
      const int row0 = m0 + q * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      st.active = row0 < args.M;
      if constexpr (EPI == kEpiResidTail) {
        // whole tiles add into the residual stream; a tail tile's part
        // stores its sums in the parts region, rows counted from tail_row0
        if (w.tail)
          epilogue_tile<EPI, BN>(args, &tmOut2, st, t_row, row0, row0 + lane, n0, hc,
                                 w.part * args.split_rows - args.tail_row0, false, w.part == 0);
        else
          epilogue_tile<EPI, BN>(args, &tmOut, st, t_row, row0, row0 + lane, n0, hc, 0, true, true);
      } else {
        epilogue_tile<EPI, BN>(args, &tmOut, st, t_row, row0, row0 + lane, n0, hc,
                               EPI == kEpiPartial ? w.part * args.split_rows : 0, EPI == kEpiResid,
                               EPI == kEpiResid || (EPI == kEpiPartial && w.part == 0));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      acc ^= 1;
      if (acc == 0) aphase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // no CTA of the pair leaves while the other may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, C::TMEM_COLS);
  }
}

template <int EPI, int BN>
cudaError_t launch_one(const GemmMaps& m, const GemmArgs& args, int num_sms, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_tc_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Cfg<BN>::SMEM));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int num_tiles = ((args.M + BM - 1) / BM) * (args.N / BN);
  if (num_tiles == 0) return cudaSuccess;
  const int num_units = EPI == kEpiPartial    ? num_tiles * args.splits
                        : EPI == kEpiResidTail ? args.main_tiles + (num_tiles - args.main_tiles) * args.splits
                                               : num_tiles;
  const int max_clusters = num_sms / 2;
  const int clusters = num_units < max_clusters ? num_units : max_clusters;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  return launch_pdl(gemm_tc_kernel<EPI, BN>, dim3(2 * clusters, 1, 1), dim3(THREADS, 1, 1), Cfg<BN>::SMEM, stream,
                    attr, 1, *m.a, *m.b, *m.out, m.out2 ? *m.out2 : *m.out, args);
}

}  // namespace

cudaError_t launch_gemm(int epilogue, const GemmMaps& m, const GemmArgs& args, int num_sms, cudaStream_t stream,
                        int bn) {
  if (bn != kGemmBN && bn != kGemmBNNarrow) return cudaErrorInvalidValue;
  if (args.N % bn || args.K % BK || args.M < 0 || !m.a || !m.b || !m.out) return cudaErrorInvalidValue;
  if (epilogue == kEpiPartial &&
      (bn != kGemmBN || args.splits < 1 || args.splits > args.K / BK || args.split_rows % BM ||
       args.split_rows < ((args.M + BM - 1) / BM) * BM))
    return cudaErrorInvalidValue;
  if (epilogue == kEpiResidTail) {
    // whole row blocks before the tail, parts that fit the parts region (a
    // bias is added by whole tiles and by part 0 of the split ones)
    const int num_n = args.N / bn, num_tiles = ((args.M + BM - 1) / BM) * num_n;
    if (bn != kGemmBN || !m.out2 || args.splits < 1 || args.splits > args.K / BK ||
        args.main_tiles < 0 || args.main_tiles >= num_tiles || args.main_tiles % num_n ||
        args.tail_row0 != (args.main_tiles / num_n) * BM || args.split_rows % BM ||
        args.split_rows < ((args.M - args.tail_row0 + BM - 1) / BM) * BM)
      return cudaErrorInvalidValue;
  }
  if (bn == kGemmBNNarrow) {
    // narrow 256 x 128 tiles: twice the tiles per wave, for small M where a
    // GEMM's 256-column tiles leave most clusters idle
    switch (epilogue) {
      case kEpiQkvRope: return launch_one<kEpiQkvRope, kGemmBNNarrow>(m, args, num_sms, stream);
      case kEpiQkvBias: return launch_one<kEpiQkvBias, kGemmBNNarrow>(m, args, num_sms, stream);
      case kEpiResid: return launch_one<kEpiResid, kGemmBNNarrow>(m, args, num_sms, stream);
      case kEpiGeglu: return launch_one<kEpiGeglu, kGemmBNNarrow>(m, args, num_sms, stream);
      case kEpiBiasRelu: return launch_one<kEpiBiasRelu, kGemmBNNarrow>(m, args, num_sms, stream);
      case kEpiStoreF32: return launch_one<kEpiStoreF32, kGemmBNNarrow>(m, args, num_sms, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (epilogue) {
    case kEpiQkvRope: return launch_one<kEpiQkvRope, kGemmBN>(m, args, num_sms, stream);
    case kEpiQkvBias: return launch_one<kEpiQkvBias, kGemmBN>(m, args, num_sms, stream);
    case kEpiResid: return launch_one<kEpiResid, kGemmBN>(m, args, num_sms, stream);
    case kEpiGeglu: return launch_one<kEpiGeglu, kGemmBN>(m, args, num_sms, stream);
    case kEpiBiasRelu: return launch_one<kEpiBiasRelu, kGemmBN>(m, args, num_sms, stream);
    case kEpiScorer: return launch_one<kEpiScorer, kGemmBN>(m, args, num_sms, stream);
    case kEpiStoreF32: return launch_one<kEpiStoreF32, kGemmBN>(m, args, num_sms, stream);
    case kEpiPartial: return launch_one<kEpiPartial, kGemmBN>(m, args, num_sms, stream);
    case kEpiResidTail: return launch_one<kEpiResidTail, kGemmBN>(m, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ---- tensor maps -------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, bool f32, uint64_t rows, uint64_t cols, uint32_t box_cols,
                 uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  const uint64_t es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (cols * es) % 16 || box_cols * es != 128 || rows == 0) return -2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * es};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k, uint32_t box_rows) {
  if (k % 64) return -2;
  return make_tmap_2d(map, base, false, rows, k, 64, box_rows);
}

}  // namespace laya
