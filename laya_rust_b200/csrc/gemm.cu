// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
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
// CTA = 6 warps, one CTA per SM, persistent over 128x256 output tiles:
//   warp 0      TMA producer: A 128x64 and W 256x64 tiles, 128B swizzle,
//               into a 4-stage shared-memory ring (48 KB per stage)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=256, K=16 per instruction), accumulators in TMEM,
//               double-buffered (2 x 256 columns) so the epilogue of tile i
//               overlaps the main loop of tile i+1
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, fused math,
//               global stores; warp w reads TMEM lanes 32*(w%4)..+31
// No clusters and no multicast: every CTA loads its own tiles.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int BM = kGemmBM, BN = kGemmBN, BK = kGemmBK;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;
constexpr int BAR_BYTES = 256;
constexpr size_t SMEM_BYTES = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + BAR_BYTES;

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Stores 32 f16 values (packed in 16 words) to 64 contiguous bytes.
__device__ __forceinline__ void store_32h(__half* dst, const uint32_t (&p)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
}

template <int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, uint32_t t_row, int row, int n0) {
  const bool valid = row < a.M;
  if constexpr (EPI == kEpiQkvRope) {
    const int part = n0 / 1024;
    __half* out = static_cast<__half*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + n0;
    if (part < 2) {
      float cs[32], sn[32];
      const int p = valid ? a.pos[row] : 0;
      const float4* c4 = reinterpret_cast<const float4*>(a.cosb + p * 32);
      const float4* s4 = reinterpret_cast<const float4*>(a.sinb + p * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 c = __ldg(c4 + i), s = __ldg(s4 + i);
        cs[4 * i] = c.x; cs[4 * i + 1] = c.y; cs[4 * i + 2] = c.z; cs[4 * i + 3] = c.w;
        sn[4 * i] = s.x; sn[4 * i + 1] = s.y; sn[4 * i + 2] = s.z; sn[4 * i + 3] = s.w;
      }
#pragma unroll 1
      for (int hh = 0; hh < BN / 64; ++hh) {
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(t_row + hh * 64, lo);
        tmem_ld_32x32b_x32(t_row + hh * 64 + 32, hi);
        tmem_ld_wait();
        uint32_t plo[16], phi[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          // rotate-half RoPE: d < 32: q*c - q[d+32]*s ; d >= 32: q*c + q[d-32]*s
          float a0 = u2f(lo[j]), b0 = u2f(hi[j]), a1 = u2f(lo[j + 1]), b1 = u2f(hi[j + 1]);
          float r0 = (a0 * cs[j] - b0 * sn[j]) * a.scale;
          float r1 = (a1 * cs[j + 1] - b1 * sn[j + 1]) * a.scale;
          float s0 = (b0 * cs[j] + a0 * sn[j]) * a.scale;
          float s1 = (b1 * cs[j + 1] + a1 * sn[j + 1]) * a.scale;
          plo[j / 2] = pack_half2(r0, r1);
          phi[j / 2] = pack_half2(s0, s1);
        }
        if (valid) {
          store_32h(out + hh * 64, plo);
          store_32h(out + hh * 64 + 32, phi);
        }
      }
    } else {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + c0, v);
        tmem_ld_wait();
        uint32_t p[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) p[j / 2] = pack_half2(u2f(v[j]), u2f(v[j + 1]));
        if (valid) store_32h(out + c0, p);
      }
    }
  } else if constexpr (EPI == kEpiQkvBias) {
    const int part = n0 / 1024;
    const float sc = part < 2 ? a.scale : 1.0f;
    __half* out = static_cast<__half*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + n0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      uint32_t p[16];
      const float* b = a.bias + n0 + c0;
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        p[j / 2] = pack_half2((u2f(v[j]) + __ldg(b + j)) * sc, (u2f(v[j + 1]) + __ldg(b + j + 1)) * sc);
      if (valid) store_32h(out + c0, p);
    }
  } else if constexpr (EPI == kEpiResid) {
    float* x = static_cast<float*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + n0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      if (valid) {
        float4* xp = reinterpret_cast<float4*>(x + c0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 o = xp[i];
          float p0 = u2f(v[4 * i]), p1 = u2f(v[4 * i + 1]), p2 = u2f(v[4 * i + 2]),
                p3 = u2f(v[4 * i + 3]);
          if (a.bias) {
            const float* b = a.bias + n0 + c0 + 4 * i;
            p0 += __ldg(b); p1 += __ldg(b + 1); p2 += __ldg(b + 2); p3 += __ldg(b + 3);
          }
          o.x += p0; o.y += p1; o.z += p2; o.w += p3;
          xp[i] = o;
        }
      }
    }
  } else if constexpr (EPI == kEpiGeglu) {
    const int oc0 = (n0 / BN) * (BN / 2);
    __half* out = static_cast<__half*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + oc0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN / 2; c0 += 32) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(t_row + c0, g);
      tmem_ld_32x32b_x32(t_row + BN / 2 + c0, u);
      tmem_ld_wait();
      if (oc0 + c0 >= a.n_valid) continue;
      uint32_t p[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        p[j / 2] = pack_half2(gelu_erf(u2f(g[j])) * u2f(u[j]), gelu_erf(u2f(g[j + 1])) * u2f(u[j + 1]));
      if (valid) store_32h(out + c0, p);
    }
  } else if constexpr (EPI == kEpiBiasRelu) {
    __half* out = static_cast<__half*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + n0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      uint32_t p[16];
      const float* b = a.bias + n0 + c0;
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        p[j / 2] = pack_half2(fmaxf(u2f(v[j]) + __ldg(b + j), 0.0f),
                              fmaxf(u2f(v[j + 1]) + __ldg(b + j + 1), 0.0f));
      if (valid) store_32h(out + c0, p);
    }
  } else if constexpr (EPI == kEpiScorer) {
    float s = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      const float* b = a.bias + n0 + c0;
      const float* w = a.wvec + n0 + c0;
#pragma unroll
      for (int j = 0; j < 32; ++j) s += gelu_erf(u2f(v[j]) + __ldg(b + j)) * __ldg(w + j);
    }
    if (valid) static_cast<float*>(a.out)[static_cast<size_t>(n0 / BN) * a.ldo + row] = s;
  } else {  // kEpiStoreF32
    float* out = static_cast<float*>(a.out) + static_cast<size_t>(valid ? row : 0) * a.ldo + n0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c0, v);
      tmem_ld_wait();
      if (valid) {
        float4* o = reinterpret_cast<float4*>(out + c0);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          o[i] = make_float4(u2f(v[4 * i]), u2f(v[4 * i + 1]), u2f(v[4 * i + 2]), u2f(v[4 * i + 3]));
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (args.M + BM - 1) / BM;
  const int num_n = args.N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = args.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[STAGES];
      uint32_t issued_mask = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % num_m) * BM;
        const int n0 = (tile / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, args.err, kErrGemmProducerWait,
                                 abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, m0, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &tmB, kb * BK, n0, &full[stage]);
          issued_parity[stage] = phase;
          issued_mask |= 1u << stage;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Let every load this thread issued land before the CTA can exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_wait_bounded(&full[s], issued_parity[s], args.err, kErrGemmTeardownWait, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait_bounded(&tempty[acc], aphase ^ 1u, args.err, kErrGemmMmaWait, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, args.err, kErrGemmMmaWait, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                     idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aphase ^= 1u;
      }
      // Every MMA issued by this thread completes before TMEM is released.
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, args.err, kErrGemmTeardownWait, nullptr);
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_bounded(&tfull[acc], aphase, args.err, kErrGemmEpilogueWait, abort_flag);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * BM;
      const int n0 = (tile / num_m) * BN;
      const int row = m0 + q * 32 + lane;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      epilogue_tile<EPI>(args, t_row, row, n0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aphase ^= 1u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int EPI>
cudaError_t launch_one(const CUtensorMap* tmA, const CUtensorMap* tmB, const GemmArgs& args,
                       int num_sms, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int num_tiles = ((args.M + BM - 1) / BM) * (args.N / BN);
  if (num_tiles == 0) return cudaSuccess;
  const int grid = num_tiles < num_sms ? num_tiles : num_sms;
  gemm_tc_kernel<EPI><<<grid, THREADS, SMEM_BYTES, stream>>>(*tmA, *tmB, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(int epilogue, const CUtensorMap* tmA, const CUtensorMap* tmB,
                        const GemmArgs& args, int num_sms, cudaStream_t stream) {
  if (args.N % BN || args.K % BK || args.M < 0) return cudaErrorInvalidValue;
  switch (epilogue) {
    case kEpiQkvRope: return launch_one<kEpiQkvRope>(tmA, tmB, args, num_sms, stream);
    case kEpiQkvBias: return launch_one<kEpiQkvBias>(tmA, tmB, args, num_sms, stream);
    case kEpiResid: return launch_one<kEpiResid>(tmA, tmB, args, num_sms, stream);
    case kEpiGeglu: return launch_one<kEpiGeglu>(tmA, tmB, args, num_sms, stream);
    case kEpiBiasRelu: return launch_one<kEpiBiasRelu>(tmA, tmB, args, num_sms, stream);
    case kEpiScorer: return launch_one<kEpiScorer>(tmA, tmB, args, num_sms, stream);
    case kEpiStoreF32: return launch_one<kEpiStoreF32>(tmA, tmB, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ---- tensor maps -------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k,
                  uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (k * 2) % 16 || k % 64) return -2;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {k * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

}  // namespace laya
