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

constexpr int CHUNK = 256;    // features one pass of the 32 lanes covers (8 each)

__device__ __forceinline__ float load1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }
__device__ __forceinline__ float load1(const __half* p) { return __half2float(p[0]); }

// code_logits: one warp per work item of PW prompts x CW codes (CW = 4, 8 or 16 by the number of codes), 4 warps a
// CTA. The items of a CTA share their codes, so a code row is read from L2 once per CTA and from L1 by its other warps;
// at the C4 sizes (R = 256, up to 255 codes: 1,024 warps) every item is resident at once. The 32 lanes split the
// features: lane l takes l * 8 .. l * 8 + 7 of every 256-feature chunk (16-byte loads), in increasing order, then the
// ragged tail (every feature, when a row does not start on a 16-byte boundary) lane-strided (l, l + 32, ...); so a
// warp holds every feature of its dot products and no partial sum crosses warps. The 32 lane partials of each value
// are then added in a fixed pairing (lanes l and l ^ 16, then ^ 8, ^ 4, ^ 2, ^ 1) by recursive halving: at distance d
// a lane keeps half of its values and adds its partner's copy of that half, so only PW * CW / 32 values a lane remain
// at the end instead of PW * CW all-lane trees. Every z[r, u] is therefore one fixed function of h[r, :], the code's
// row and D: a prompt's logits do not depend on the other prompts or codes of the call (the contract of
// CodeReadout.probs_each, readout.py:86-104).
constexpr int PW = 4;         // prompts a warp item
constexpr int IWARPS = 4;     // warps (items) a CTA

template <int NV>
__device__ __forceinline__ void halving_reduce(float (&v)[NV], int lane) {
  int cnt = NV;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    if (cnt >= 2) {
      const int half = cnt / 2;
      const bool up = (lane & d) != 0;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        if (i < half) {
          const float send = up ? v[i] : v[i + half];
          const float keep = up ? v[i + half] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, d));
        }
      }
      cnt = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], d));
    }
  }
}

template <typename TH, typename TW, typename TB, int CW>
__global__ void __launch_bounds__(IWARPS * 32) code_logits_warp_kernel(
    const TH* __restrict__ h, int64_t R, int64_t D, int64_t ldh, const TW* __restrict__ head, int64_t V, int64_t ldw,
    const int64_t* __restrict__ ids, int64_t U, const TB* __restrict__ bias, float softcap, float* __restrict__ z) {
  constexpr int NV = PW * CW;                   // values of a warp item (16, 32 or 64)
  constexpr int PER = NV >= 32 ? NV / 32 : 1;   // values a lane keeps after the reduction
  constexpr int REP = NV >= 32 ? 1 : 32 / NV;   // lanes that hold each value (NV < 32)
  pdl_launch();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pgroups = (R + PW - 1) / PW;
  const int64_t item = (int64_t)blockIdx.x * IWARPS + warp;
  const int64_t cb = item / pgroups, pg = item - cb * pgroups;
  if (cb * CW >= U) return;  // past the last item (whole warps only)
  const int64_t r0 = pg * PW, u0 = cb * CW;
  int64_t myid = -1;  // lane j < CW: the id of code u0 + j (-1: past U or out of range)
  if (lane < CW && u0 + lane < U) {
    const int64_t id = __ldg(ids + u0 + lane);
    const bool ok = id >= 0 && id < V;
    if (!ok && pg == 0) atomicOr(&g_fault, kFaultBadId);
    myid = ok ? id : -1;
  }
  int64_t hoff[PW], woff[CW];  // element offsets of the rows (a row past R or a bad id reads row 0)
#pragma unroll
  for (int i = 0; i < PW; ++i) hoff[i] = r0 + i < R ? (r0 + i) * ldh : 0;
#pragma unroll
  for (int j = 0; j < CW; ++j) {
    const int64_t id = __shfl_sync(0xffffffffu, myid, j);
    woff[j] = id >= 0 ? id * ldw : 0;
  }
  float acc[NV];
#pragma unroll
  for (int e = 0; e < NV; ++e) acc[e] = 0.0f;
  const bool vec = ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(head)) & 15) == 0 &&
                   (ldh * (int64_t)sizeof(TH)) % 16 == 0 && (ldw * (int64_t)sizeof(TW)) % 16 == 0;
  const int64_t dv = vec ? D / CHUNK * CHUNK : 0;
  for (int64_t d = lane * 8; d < dv; d += CHUNK) {
    float a[PW][8], b[8];
#pragma unroll
    for (int i = 0; i < PW; ++i) load8(h + hoff[i] + d, a[i]);
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      load8(head + woff[j] + d, b);
#pragma unroll
      for (int i = 0; i < PW; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i * CW + j] = fmaf(a[i][e], b[e], acc[i * CW + j]);
    }
  }
  for (int64_t d = dv + lane; d < D; d += 32) {
    float a[PW];
#pragma unroll
    for (int i = 0; i < PW; ++i) a[i] = load1(h + hoff[i] + d);
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      const float b = load1(head + woff[j] + d);
#pragma unroll
      for (int i = 0; i < PW; ++i) acc[i * CW + j] = fmaf(a[i], b, acc[i * CW + j]);
    }
  }
  halving_reduce<NV>(acc, lane);
  // value e = i * CW + j now sits in lane e / PER, slot e % PER (NV >= 32), or in lanes e * REP .. (NV < 32)
  int64_t eid[PER];  // the id of each kept value's code (-1: none)
#pragma unroll
  for (int k = 0; k < PER; ++k) eid[k] = __shfl_sync(0xffffffffu, myid, ((lane / REP) * PER + k) % CW);
  if (lane % REP == 0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int e = (lane / REP) * PER + k;
      const int i = e / CW, j = e % CW;
      const int64_t r = r0 + i, u = u0 + j;
      if (r < R && u < U) {
        float v = acc[k];
        if (eid[k] < 0) {
          v = __int_as_float(0x7fc00000);
        } else if (bias) {
          v = __fadd_rn(v, load1(bias + eid[k]));
        }
        if (softcap > 0.0f) v = __fmul_rn(tanhf(__fdiv_rn(v, softcap)), softcap);
        z[r * U + u] = v;
      }
    }
  }
}

// One warp per prompt row, NI <= 32 codes a lane (Kmax <= 32 NI): every index, padding flag and logit is loaded
// before any arithmetic (one round trip each), then max, exp, sum and division in the same order for every NI.
template <int NI>
__global__ void __launch_bounds__(256) code_probs_kernel(const float* __restrict__ z, int64_t R, int64_t U,
                                                         const int64_t* __restrict__ idx,
                                                         const uint8_t* __restrict__ pad, int64_t Kmax,
                                                         float* __restrict__ p) {
  pdl_launch();
  pdl_wait();
  const int64_t r = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  int64_t c[NI];
  bool use[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int64_t j = lane + 32 * i;
    const bool in = j < Kmax;
    c[i] = in ? __ldg(idx + r * Kmax + j) : -1;
    use[i] = in && !(pad && __ldg(pad + r * Kmax + j));
  }
  float v[NI];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    v[i] = (use[i] && c[i] >= 0 && c[i] < U) ? z[r * U + c[i]] : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    v[i] = (v[i] == -INFINITY) ? 0.0f : expf(__fsub_rn(v[i], m));
    s = __fadd_rn(s, v[i]);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int64_t j = lane + 32 * i;
    if (j < Kmax) p[r * Kmax + j] = __fdiv_rn(v[i], s);
  }
}

}  // namespace readout
}  // namespace b200
