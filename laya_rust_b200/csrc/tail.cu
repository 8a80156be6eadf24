// The decision tail: scorer output sum, marker post-processing and the act
// head, one cluster of kSplit CTAs per sequence.
//
// Reference semantics (laya-rust): scorer output projection + bias
// (graph.rs:166-167), post (backend/cpu/mod.rs:400-451: logits masked to
// -10000 where mmask == 0, softmax over all k markers, features
// [top1, top1 - top2, entropy / ln(max(nv,2)), max(nv,2) / 255]), act_input
// (:453-465: the sequence's first row ++ features), act MLP
// (graph.rs:171-176: W1 [256,1028] + b1, GELU, W2 [2,256] + b2).
// The 1024 -> 1024 scorer hidden layer runs in the GEMM (kEpiScorer), which
// leaves one partial dot product per 128 output columns; they are summed here
// in a fixed order.
//
// CTA c of a sequence's cluster computes the act input (every CTA: the CLS row
// and the four post features) and hidden units [32c, 32c + 32) from W1's
// rows there, so the 526 KB of W1 are read by kSplit CTAs, 66 KB each, not
// all by one.  After a cluster barrier CTA 0 reads the other CTAs' hidden
// units from their shared memory (distributed shared memory) and applies W2
// in the same order as a single CTA would; it alone writes the logits.
#include "common.cuh"
#include "kernels.h"

namespace laya {

namespace {

constexpr int HID = 1024;
constexpr int AIN = HID + 4;
constexpr int AH = 256;
constexpr int kRowsPerPass = 4;  // W1 rows a warp reads together
constexpr int kSplit = 8;        // CTAs (a cluster) per sequence
constexpr int kHidPerCta = AH / kSplit;
constexpr int kTailThreads = 32 * (kHidPerCta / kRowsPerPass);  // one pass: 8 warps x 4 rows
static_assert(AIN % 4 == 0 && kHidPerCta % kRowsPerPass == 0, "act head tiling");

__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// a float in CTA `rank`'s shared memory at the address of `p` in this CTA's
__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
  uint32_t a, r;
  a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kTailThreads) tail_kernel(const TailArgs a) {
  extern __shared__ float sm[];
  float* ain = sm;             // [1028]
  float* hid = sm + AIN;       // [32]: this CTA's hidden units
  float* lg = hid + kHidPerCta;  // [k]
  grid_dep_wait();
  grid_dep_trigger();
  const int b = blockIdx.x;
  const uint32_t crank = cta_rank_in_cluster();  // == blockIdx.y
  const int k = a.k;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  for (int j = tid; j < k; j += blockDim.x) {
    const int r = b * k + j;
    float v;
    if (a.mmask[r] != 0) {
      v = a.partial[r];
      for (int nt = 1; nt < kScorerPartials; ++nt) v += a.partial[static_cast<size_t>(nt) * a.ldp + r];
      v += a.score_bias;
    } else {
      v = -10000.0f;
    }
    lg[j] = v;
    if (crank == 0) a.logits[r] = v;
  }
  const float* xc = a.x + static_cast<size_t>(a.cls_row[b]) * HID;
  for (int i = tid; i < HID; i += blockDim.x) ain[i] = xc[i];
  __syncthreads();
  if (tid == 0) {
    float mx = -3.4e38f;
    for (int j = 0; j < k; ++j) mx = fmaxf(mx, lg[j]);
    float sum = 0.0f;
    for (int j = 0; j < k; ++j) sum += expf(lg[j] - mx);
    const float inv = 1.0f / sum;
    float t1 = -1.0f, t2 = -1.0f, ent = 0.0f;
    int nv = 0;
    for (int j = 0; j < k; ++j) {
      const float p = expf(lg[j] - mx) * inv;
      if (p > t1) {
        t2 = t1;
        t1 = p;
      } else if (p > t2) {
        t2 = p;
      }
      ent -= p * logf(fmaxf(p, 1e-9f));
      if (a.mmask[b * k + j] != 0) ++nv;
    }
    if (t2 < 0.0f) t2 = 0.0f;
    const float nn = static_cast<float>(nv < 2 ? 2 : nv);
    ain[HID] = t1;
    ain[HID + 1] = t1 - t2;
    ain[HID + 2] = ent / logf(nn);
    ain[HID + 3] = nn / 255.0f;
  }
  __syncthreads();
  // act hidden layer: each warp takes kRowsPerPass rows of W1 at a time and
  // loads all of them (8-byte pieces: a row is 2056 bytes, 8-byte aligned)
  // before it sums, so a warp has kRowsPerPass x 9 loads in flight instead
  // of one row's dependent chain
  const int nwarps = blockDim.x >> 5;
  for (int o0 = static_cast<int>(crank) * kHidPerCta + warp * kRowsPerPass; o0 < (static_cast<int>(crank) + 1) * kHidPerCta;
       o0 += nwarps * kRowsPerPass) {
    constexpr int kIters = (AIN / 4 + 31) / 32;  // 9 pieces per lane per row
    uint2 wv[kRowsPerPass][kIters];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int i4 = lane + 32 * it;
#pragma unroll
      for (int r = 0; r < kRowsPerPass; ++r)
        wv[r][it] = i4 < AIN / 4
                        ? __ldg(reinterpret_cast<const uint2*>(a.w1 + static_cast<size_t>(o0 + r) * AIN) + i4)
                        : make_uint2(0u, 0u);
    }
    float s[kRowsPerPass];
#pragma unroll
    for (int r = 0; r < kRowsPerPass; ++r) s[r] = 0.0f;
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int i4 = lane + 32 * it;
      if (i4 < AIN / 4) {
        const float4 x = *reinterpret_cast<const float4*>(ain + 4 * i4);
#pragma unroll
        for (int r = 0; r < kRowsPerPass; ++r) {
          const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv[r][it].x));
          const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv[r][it].y));
          s[r] += w01.x * x.x + w01.y * x.y + w23.x * x.z + w23.y * x.w;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsPerPass; ++r) {
      const float t = warp_sum(s[r]);
      if (lane == 0) hid[o0 + r - static_cast<int>(crank) * kHidPerCta] = gelu_erf(t + a.b1[o0 + r]);
    }
  }
  // every CTA's hidden units written and visible across the cluster
  cluster_sync_all();
  if (crank == 0 && warp < 2) {
    // hidden unit i lives in CTA i / 32 at index i % 32
    const float* w = a.w2 + warp * AH;
    float s = 0.0f;
    for (int i = lane; i < AH; i += 32) s += w[i] * ld_cluster_f32(hid + (i % kHidPerCta), i / kHidPerCta);
    s = warp_sum(s);
    if (lane == 0) a.act[b * 2 + warp] = s + a.b2[warp];
  }
  // no CTA leaves while CTA 0 may still read its shared memory
  cluster_sync_all();
}

}  // namespace

cudaError_t launch_tail(const TailArgs& a, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  const size_t smem = sizeof(float) * (AIN + kHidPerCta + a.k);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = kSplit;
  attr[0].val.clusterDim.z = 1;
  return launch_pdl(tail_kernel, dim3(a.n, kSplit), dim3(kTailThreads), smem, s, attr, 1, a);
}

}  // namespace laya
