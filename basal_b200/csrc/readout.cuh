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
      for (int e = 0; e < 8; ++e)  // consecutive FMAs on the PW prompts' accumulators: independent, no stall
#pragma unroll
        for (int i = 0; i < PW; ++i) acc[i * CW + j] = fmaf(a[i][e], b[e], acc[i * CW + j]);
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

// code_logits for 16-bit h and head with D a multiple of 256 and many codes (U > 8): a CTA of 8 warps takes 32
// prompts x 16 codes, warp w the prompts 4w .. 4w + 3 of it. The CTA's 48 rows are staged in shared memory by bulk
// copies, 1024 features at a time in two buffers (one warp issues a row a lane), so every byte a chunk needs is
// requested at once instead of in 8 dependent rounds of register loads. A lane then walks exactly the features it
// walks in code_logits_warp_kernel (l * 8 .. l * 8 + 7 of every 256-feature chunk, in increasing order) and the
// partials meet in the same halving reduction, so every z[r, u] is the same bits whichever of the two kernels
// computes it.
constexpr int SR = 32;      // prompts a staged CTA
constexpr int SU = 16;      // codes a staged CTA
constexpr int SDC = 1024;   // features a staged chunk
constexpr int SWARPS = SR / PW;

template <typename TH, typename TW>
struct StagedSmem {
  TW w[2][SU][SDC];
  TH h[2][SR][SDC];
  uint64_t full[2];
  int abort;
};

template <typename TH, typename TW, typename TB>
__global__ void __launch_bounds__(SWARPS * 32) code_logits_staged_kernel(
    const TH* __restrict__ h, int64_t R, int64_t D, int64_t ldh, const TW* __restrict__ head, int64_t V, int64_t ldw,
    const int64_t* __restrict__ ids, int64_t U, const TB* __restrict__ bias, float softcap, float* __restrict__ z) {
  static_assert(sizeof(TH) == 2 && sizeof(TW) == 2, "16-bit rows");
  constexpr int NV = PW * SU;  // 64 values a warp
  using S = StagedSmem<TH, TW>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  S& sh = *reinterpret_cast<S*>(smem_raw);
  pdl_launch();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)blockIdx.y * SR, u0 = (int64_t)blockIdx.x * SU;
  int64_t myid = -1;  // lane j < SU: the id of code u0 + j (-1: past U or out of range)
  if (lane < SU && u0 + lane < U) {
    const int64_t id = __ldg(ids + u0 + lane);
    const bool ok = id >= 0 && id < V;
    if (!ok && blockIdx.y == 0 && warp == 0) atomicOr(&g_fault, kFaultBadId);
    myid = ok ? id : -1;
  }
  if (threadIdx.x == 0) {
    mbar_init(&sh.full[0], 1);
    mbar_init(&sh.full[1], 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int nch = (int)((D + SDC - 1) / SDC);
  // chunk c into buffer c & 1: lane l copies prompt row r0 + l and (l < SU) code row u0 + l; rows past R or without a
  // valid id copy row 0 (their results are not stored)
  auto issue = [&](int c) {
    const int b = c & 1;
    const int64_t f0 = (int64_t)c * SDC;
    const uint32_t bytes = (uint32_t)((D - f0 < SDC ? D - f0 : SDC) * 2);
    const int64_t r = r0 + lane < R ? r0 + lane : 0;
    bulk_load(sh.h[b][lane], h + r * ldh + f0, bytes, &sh.full[b]);
    if (lane < SU) bulk_load(sh.w[b][lane], head + (myid >= 0 ? myid : 0) * ldw + f0, bytes, &sh.full[b]);
    if (lane == 0) mbar_arrive_expect_tx(&sh.full[b], bytes * (SR + SU));
  };
  if (warp == 0) {
    issue(0);
    if (nch > 1) issue(1);
  }
  float acc[NV];
#pragma unroll
  for (int e = 0; e < NV; ++e) acc[e] = 0.0f;
  for (int c = 0; c < nch; ++c) {
    const int b = c & 1;
    const bool ok = mbar_wait(&sh.full[b], (uint32_t)(c >> 1) & 1, &sh.abort, kFaultTimeoutEpilogue);
    if (!__syncthreads_and(ok)) {  // a copy never landed: wait (bounded) for the ones in flight, store nothing
      if (threadIdx.x == 0) {
        blockgemm::drain_wait(&sh.full[b], (uint32_t)(c >> 1) & 1);
        if (c + 1 < nch) blockgemm::drain_wait(&sh.full[b ^ 1], (uint32_t)((c + 1) >> 1) & 1);
      }
      __syncthreads();
      return;
    }
    const int nsub = (int)((D - (int64_t)c * SDC < SDC ? D - (int64_t)c * SDC : SDC) / CHUNK);
    for (int i = 0; i < nsub; ++i) {
      const int f = i * CHUNK + lane * 8;
      float a[PW][8], bv[8];
#pragma unroll
      for (int ii = 0; ii < PW; ++ii) {
        const uint4 wv[1] = {*reinterpret_cast<const uint4*>(&sh.h[b][warp * PW + ii][f])};
        unpack8(wv, h, a[ii]);
      }
#pragma unroll
      for (int j = 0; j < SU; ++j) {
        const uint4 wv[1] = {*reinterpret_cast<const uint4*>(&sh.w[b][j][f])};
        unpack8(wv, head, bv);
#pragma unroll
        for (int e = 0; e < 8; ++e)  // consecutive FMAs on the PW prompts' accumulators: independent, no stall
#pragma unroll
          for (int ii = 0; ii < PW; ++ii) acc[ii * SU + j] = fmaf(a[ii][e], bv[e], acc[ii * SU + j]);
      }
    }
    __syncthreads();  // every warp is done with buffer b
    if (warp == 0 && c + 2 < nch) issue(c + 2);
  }
  halving_reduce<NV>(acc, lane);
  constexpr int PER = NV / 32;
  int64_t eid[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) eid[k] = __shfl_sync(0xffffffffu, myid, (lane * PER + k) % SU);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = lane * PER + k;
    const int i = e / SU, j = e % SU;
    const int64_t r = r0 + warp * PW + i, u = u0 + j;
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
