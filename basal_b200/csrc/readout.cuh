// The option-code readout (basal/readout.py:57-79) on the GPU:
//   code_logits: z[r, u] = h[r, :] . head[ids[u], :] (+ bias[ids[u]]), softcap * tanh(z / softcap) if softcap > 0,
//                the option rows gathered straight from the head (bf16 or fp32) by id, products and sums in fp32.
//                Every z[r, u] is one thread's sum over D in a fixed order, so it does not depend on the other rows
//                or codes of the batch (the contract of CodeReadout.probs_each, readout.py:86-104).
//   code_probs:  p[r, j] = softmax_j(z[r, idx[r, j]], -inf where padded), 0 at the padding (readout.py:76-79).
#pragma once
#include "quant.cuh"

namespace b200 {
namespace readout {

constexpr int TR = 16;   // prompts a CTA
constexpr int TU = 16;   // codes a CTA
constexpr int TD = 128;  // features a step

__device__ __forceinline__ float load1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }
__device__ __forceinline__ float load1(const __half* p) { return __half2float(p[0]); }

template <typename TH, typename TW, typename TB>
__global__ void __launch_bounds__(256) code_logits_kernel(const TH* __restrict__ h, int64_t R, int64_t D,
                                                          int64_t ldh, const TW* __restrict__ head, int64_t V,
                                                          int64_t ldw,
                                                          const int64_t* __restrict__ ids, int64_t U,
                                                          const TB* __restrict__ bias, float softcap,
                                                          float* __restrict__ z) {
  __shared__ float hs[TR][TD];
  __shared__ float ws[TU][TD + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t r0 = (int64_t)blockIdx.y * TR, u0 = (int64_t)blockIdx.x * TU;
  // loader role: thread t fills row t / 16 of both tiles, 8 features from (t % 16) * 8
  const int lr = threadIdx.x >> 4, lc = (threadIdx.x & 15) * 8;
  const bool hvalid = r0 + lr < R;
  const int64_t id = (u0 + lr < U) ? __ldg(ids + u0 + lr) : -1;
  const bool wvalid = id >= 0 && id < V;
  if (u0 + lr < U && !wvalid && blockIdx.y == 0 && (threadIdx.x & 15) == 0) atomicOr(&g_fault, kFaultBadId);
  const TH* hrow = h + (hvalid ? (r0 + lr) * ldh : 0);
  const TW* wrow = head + (wvalid ? id * ldw : 0);
  float acc = 0.0f;
  for (int64_t d0 = 0; d0 < D; d0 += TD) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t d = d0 + lc + i;
      hs[lr][lc + i] = (hvalid && d < D) ? load1(hrow + d) : 0.0f;
      ws[lr][lc + i] = (wvalid && d < D) ? load1(wrow + d) : 0.0f;
    }
    __syncthreads();
#pragma unroll 16
    for (int k = 0; k < TD; ++k) acc = fmaf(hs[ty][k], ws[tx][k], acc);
    __syncthreads();
  }
  const int64_t r = r0 + ty, u = u0 + tx;
  if (r < R && u < U) {
    const int64_t uid = __ldg(ids + u);
    float v = (uid >= 0 && uid < V) ? acc : __int_as_float(0x7fc00000);
    if (bias && uid >= 0 && uid < V) v = __fadd_rn(v, load1(bias + uid));
    if (softcap > 0.0f) v = __fmul_rn(tanhf(__fdiv_rn(v, softcap)), softcap);
    z[r * U + u] = v;
  }
}

// One warp per prompt row; up to 32 codes a lane.
__global__ void __launch_bounds__(256) code_probs_kernel(const float* __restrict__ z, int64_t R, int64_t U,
                                                         const int64_t* __restrict__ idx,
                                                         const uint8_t* __restrict__ pad, int64_t Kmax,
                                                         float* __restrict__ p) {
  const int64_t r = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  float v[32];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int64_t j = lane + 32 * i;
    v[i] = -INFINITY;
    if (j < Kmax && !(pad && pad[r * Kmax + j])) {
      const int64_t c = idx[r * Kmax + j];
      v[i] = (c >= 0 && c < U) ? z[r * U + c] : -INFINITY;
    }
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = (v[i] == -INFINITY) ? 0.0f : expf(__fsub_rn(v[i], m));
    s = __fadd_rn(s, v[i]);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int64_t j = lane + 32 * i;
    if (j < Kmax) p[r * Kmax + j] = __fdiv_rn(v[i], s);
  }
}

}  // namespace readout
}  // namespace b200
