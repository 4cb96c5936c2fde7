// The option-code readout (basal/readout.py:57-79) on the GPU:
//   code_logits: z[r, u] = h[r, :] . head[ids[u], :] (+ bias[ids[u]]), softcap * tanh(z / softcap) if softcap > 0,
//                the option rows gathered straight from the head (bf16 or fp32) by id, products and sums in fp32.
//                Every z[r, u] is summed in one fixed order that depends on D only, so it does not depend on the
//                other rows or codes of the batch (the contract of CodeReadout.probs_each, readout.py:86-104).
//   code_probs:  p[r, j] = softmax_j(z[r, idx[r, j]], -inf where padded), 0 at the padding (readout.py:76-79).
#pragma once
#include "quant.cuh"

namespace b200 {
namespace readout {

constexpr int WR = 4;         // prompts a CTA
constexpr int WU = 8;         // codes a CTA
constexpr int WARPS = 8;      // warps a CTA, splitting the features
constexpr int TR = WR;
constexpr int TU = WU;
constexpr int CHUNK = 256;    // features one pass of the 32 lanes covers (8 each)

__device__ __forceinline__ float load1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }
__device__ __forceinline__ float load1(const __half* p) { return __half2float(p[0]); }

// A CTA computes a 4 x 8 block of z (4 prompts x 8 codes); its 8 warps split the features, so the whole dot products
// are loaded at once (one round trip to memory): warp w takes the 256-feature chunks w, w + 8, ..., lane l the
// features l * 8 .. l * 8 + 7 of each (4 + 8 loads of 16 bytes feed 32 x 8 FMAs), summed in increasing feature order;
// the features past the last whole chunk (every feature, when a row does not start on a 16-byte boundary) go to warp
// 0, one per lane (l, l + 32, ...). The 32 lane partials of a warp are added in a fixed tree (xor 16, 8, 4, 2, 1) and
// the 8 warp partials in warp order. So every z[r, u] is one fixed function of h[r, :] and head[ids[u], :] for a given
// D: a prompt's logits do not depend on the other prompts or codes of the call (the contract of
// CodeReadout.probs_each, readout.py:86-104).
template <typename TH, typename TW, typename TB>
__global__ void __launch_bounds__(WARPS * 32) code_logits_kernel(const TH* __restrict__ h, int64_t R, int64_t D,
                                                                 int64_t ldh, const TW* __restrict__ head, int64_t V,
                                                                 int64_t ldw, const int64_t* __restrict__ ids,
                                                                 int64_t U, const TB* __restrict__ bias,
                                                                 float softcap, float* __restrict__ z) {
  __shared__ float part[WARPS][WR * WU];
  __shared__ int64_t sid[WU];
  pdl_launch();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)blockIdx.y * TR;
  const int64_t u0 = (int64_t)blockIdx.x * TU;
  if (threadIdx.x < WU) {
    const int64_t u = u0 + threadIdx.x;
    const int64_t id = u < U ? __ldg(ids + u) : -1;
    const bool ok = id >= 0 && id < V;
    if (u < U && !ok && blockIdx.y == 0) atomicOr(&g_fault, kFaultBadId);
    sid[threadIdx.x] = ok ? id : -1;
  }
  __syncthreads();
  int64_t hoff[WR], woff[WU];  // element offsets of the rows (a row past R or a bad id reads row 0)
#pragma unroll
  for (int i = 0; i < WR; ++i) hoff[i] = r0 + i < R ? (r0 + i) * ldh : 0;
#pragma unroll
  for (int j = 0; j < WU; ++j) woff[j] = sid[j] >= 0 ? sid[j] * ldw : 0;
  float acc[WR][WU];
#pragma unroll
  for (int i = 0; i < WR; ++i)
#pragma unroll
    for (int j = 0; j < WU; ++j) acc[i][j] = 0.0f;
  const bool vec = ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(head)) & 15) == 0 &&
                   (ldh * (int64_t)sizeof(TH)) % 16 == 0 && (ldw * (int64_t)sizeof(TW)) % 16 == 0;
  const int64_t dv = vec ? D / CHUNK * CHUNK : 0;
  for (int64_t d = warp * CHUNK + lane * 8; d < dv; d += WARPS * CHUNK) {
    float a[WR][8], b[8];
#pragma unroll
    for (int i = 0; i < WR; ++i) load8(h + hoff[i] + d, a[i]);
#pragma unroll
    for (int j = 0; j < WU; ++j) {
      load8(head + woff[j] + d, b);
#pragma unroll
      for (int i = 0; i < WR; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][j] = fmaf(a[i][e], b[e], acc[i][j]);
    }
  }
  if (warp == 0) {
    for (int64_t d = dv + lane; d < D; d += 32) {
      float a[WR];
#pragma unroll
      for (int i = 0; i < WR; ++i) a[i] = load1(h + hoff[i] + d);
#pragma unroll
      for (int j = 0; j < WU; ++j) {
        const float b = load1(head + woff[j] + d);
#pragma unroll
        for (int i = 0; i < WR; ++i) acc[i][j] = fmaf(a[i], b, acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < WR; ++i)
#pragma unroll
    for (int j = 0; j < WU; ++j) {
      float v = acc[i][j];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == i * WU + j) part[warp][i * WU + j] = v;  // every lane holds the same sum after the tree
    }
  __syncthreads();
  if (threadIdx.x < WR * WU) {
    const int i = threadIdx.x / WU, j = threadIdx.x % WU;
    const int64_t r = r0 + i, u = u0 + j;
    if (r < R && u < U) {
      float v = part[0][threadIdx.x];
#pragma unroll
      for (int w = 1; w < WARPS; ++w) v = __fadd_rn(v, part[w][threadIdx.x]);
      if (sid[j] < 0) v = __int_as_float(0x7fc00000);
      if (bias && sid[j] >= 0) v = __fadd_rn(v, load1(bias + sid[j]));
      if (softcap > 0.0f) v = __fmul_rn(tanhf(__fdiv_rn(v, softcap)), softcap);
      z[r * U + u] = v;
    }
  }
}

// One warp per prompt row; up to 32 codes a lane.
__global__ void __launch_bounds__(256) code_probs_kernel(const float* __restrict__ z, int64_t R, int64_t U,
                                                         const int64_t* __restrict__ idx,
                                                         const uint8_t* __restrict__ pad, int64_t Kmax,
                                                         float* __restrict__ p) {
  pdl_launch();
  pdl_wait();
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
