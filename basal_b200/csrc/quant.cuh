// Quantisers of the block formats and of NVFP4, bit-exact to the reference's CPU arithmetic (rkinas/basal 2.8.1):
// every division gives the code of an IEEE round-to-nearest division (__fdiv_rn, or reciprocal products that bound the
// quotient or are checked against the code's rounding boundaries: block_codes8, e2m1_cut_distance), every product that
// the reference rounds on its own is __fmul_rn (no contraction into an FMA), casts to e4m3 round to nearest even with
// saturation at +-448 (cvt.rn.satfinite), e2m1 codes round to nearest even with saturation at 6
// (cvt.rn.satfinite.e2m1x2), int8 rounds half to even.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace b200 {

// ---- element loads: n consecutive values as fp32 (16-byte vector loads) ----
// 8 consecutive values as raw 16-byte words (one for 16-bit types, two for fp32), loaded ahead of their use so that
// a thread has several loads in flight, then widened by unpack8.
template <typename T>
__device__ __forceinline__ void raw_load8(const T* p, uint4 (&w)[sizeof(T) / 2]) {
#pragma unroll
  for (int i = 0; i < (int)(sizeof(T) / 2); ++i) w[i] = __ldg(reinterpret_cast<const uint4*>(p) + i);
}
__device__ __forceinline__ void unpack8(const uint4 (&w)[1], const __nv_bfloat16*, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w[0]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack8(const uint4 (&w)[1], const __half*, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&w[0]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack8(const uint4 (&w)[2], const float*, float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    v[4 * i] = __uint_as_float(w[i].x);
    v[4 * i + 1] = __uint_as_float(w[i].y);
    v[4 * i + 2] = __uint_as_float(w[i].z);
    v[4 * i + 3] = __uint_as_float(w[i].w);
  }
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ float e4m3_to_float(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ uint8_t float_to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// 8 values of one group -> 8 code bytes of v / sc (an IEEE division in the reference); INT8: round half to even, clamp
// to +-127, cast; FP8: cast two at a time with cvt.rn.satfinite.e4m3x2, whose saturation at +-448 is the reference's
// clamp (the quotient never exceeds 448 by more than rounding). Every code equals the one of the reference's x / s
// (checked against the oracle); the quotients are first bounded, and the lane divides its 8 values exactly only when
// the bounds leave the code open (about 1e-5 of random data):
//   INT8: y = v * RN(1 / sc) is within 1.5 ulp of the correctly rounded quotient, so it gives the same code unless
//   some y lies within a few ulps of a half-integer.
//   FP8: lo = RZ(v * RD(1 / sc)) and hi = RU(|v| * RU(1 / sc)) bracket |v / sc| (|lo| <= |v / sc| <= hi), hence
//   also its correctly rounded value; the e4m3 cast is monotone in magnitude, so equal codes of |lo| and hi are the
//   code's magnitude, and lo carries the sign (a -0 included). RD / RU (1 / sc) come from r = RN(1 / sc) and the sign
//   of 1 - r sc (one fma): r itself on one side, its neighbour float on the other.
// ---------------------------------------------------------------------------------------------------------------
template <bool INT8>
__device__ __forceinline__ uint2 block_codes8(const float (&v)[8], float sc) {
  const float rcp = __frcp_rn(sc);
  float y[8];
  bool near = false;
  uint32_t w[2] = {0u, 0u};
  if (INT8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      y[i] = __fmul_rn(v[i], rcp);
      near |= fabsf(__fsub_rn(y[i], __fadd_rn(floorf(y[i]), 0.5f))) < 0x1p-14f;
    }
  } else {
    const float e = __fmaf_rn(-rcp, sc, 1.0f);  // its sign is that of 1 / sc - rcp (NaN for sc = inf: rcp = 0 kept)
    const uint32_t rb = __float_as_uint(rcp);
    const float rlo = e < 0.0f ? __uint_as_float(rb - 1u) : rcp;
    const float rhi = e > 0.0f ? __uint_as_float(rb + 1u) : rcp;
    uint32_t diff = 0u;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const uint32_t lo = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
          make_float2(__fmul_rz(v[i], rlo), __fmul_rz(v[i + 1], rlo)), __NV_SATFINITE, __NV_E4M3));
      const uint32_t hi = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
          make_float2(__fmul_ru(fabsf(v[i]), rhi), __fmul_ru(fabsf(v[i + 1]), rhi)), __NV_SATFINITE, __NV_E4M3));
      diff |= (lo & 0x7F7Fu) ^ hi;
      w[i >> 2] |= lo << (8 * (i & 3));
    }
    if (diff == 0u) return make_uint2(w[0], w[1]);
    near = true;
    w[0] = w[1] = 0u;
  }
  if (near) {
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fdiv_rn(v[i], sc);
  }
  if (INT8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t = fminf(fmaxf(rintf(y[i]), -127.0f), 127.0f);
      const uint32_t b = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(__float2int_rn(t))));
      w[i >> 2] |= b << (8 * (i & 3));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const uint32_t b =
          static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(y[i], y[i + 1]), __NV_SATFINITE, __NV_E4M3));
      w[i >> 2] |= b << (8 * (i & 3));
    }
  }
  return make_uint2(w[0], w[1]);
}

// ---------------------------------------------------------------------------------------------------------------
// Activations, FP8 / INT8 block formats: one half-warp per 128-feature group (8 values a lane), amax by shuffles; a
// warp loads PAIRS pairs of groups before it computes any (1 for a few rows, where fewer, longer warps cost latency;
// enough groups to fill the GPU take act_quant_wide_kernel below).
// basal/blockquant.py:118-123: s = max(amax, 1e-12) / qmax; q = cast(clamp(x / s)) (INT8: round first). The
// activations are contiguous, so group g is the 128 values from element 128 g. (Measured on B200: this kernel is
// bound by its per-value arithmetic, not by bytes in flight; staging chunks through shared memory did not speed it.)
// ---------------------------------------------------------------------------------------------------------------
template <typename T, bool INT8, int PAIRS>
__global__ void __launch_bounds__(256) act_quant_block_kernel(const T* __restrict__ x, int64_t groups,
                                                              uint8_t* __restrict__ q, float* __restrict__ s,
                                                              int early) {
  if (early) pdl_launch();  // one resident wave: the next kernel's set-up may overlap all of this grid
  pdl_wait();
  constexpr float kQmax = INT8 ? 127.0f : 448.0f;
  constexpr int W = sizeof(T) / 2;  // 16-byte words of a lane's 8 values
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, l = lane & 15;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t p = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * PAIRS; 2 * p < groups;
       p += warps * PAIRS) {
    // all the loads of the warp's PAIRS group pairs first (HBM wants bytes in flight), then the arithmetic
    uint4 w[PAIRS][W];
#pragma unroll
    for (int u = 0; u < PAIRS; ++u) {
      const int64_t g = 2 * (p + u) + half;
      if (g < groups) {
        raw_load8(x + g * 128 + l * 8, w[u]);
      } else {
#pragma unroll
        for (int i = 0; i < W; ++i) w[u][i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = 0; u < PAIRS; ++u) {
      const int64_t g = 2 * (p + u) + half;
      float v[8];
      unpack8(w[u], x, v);
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), kQmax);
      const uint2 codes = block_codes8<INT8>(v, sc);
      if (g < groups) {
        *reinterpret_cast<uint2*>(q + g * 128 + l * 8) = codes;
        if (l == 0) s[g] = sc;
      }
    }
  }
  // else the next kernel (a GEMM whose CTAs each fill an SM while they wait for this grid) may launch once every
  // CTA here has done its work: triggered at the start, its CTAs took the SMs from this grid's later waves
  if (!early) pdl_launch();
}

// The same quantiser for many groups: LPG lanes a group (128 / LPG values a lane, contiguous), 32 / LPG groups a warp
// step, the loads of U steps issued before any arithmetic. Its per-group work (the shuffles, the scale's division and
// reciprocal) is shared by more values a lane; the codes are the same as act_quant_block_kernel's.
template <typename T, bool INT8, int U, int LPG>
__global__ void __launch_bounds__(256) act_quant_wide_kernel(const T* __restrict__ x, int64_t groups,
                                                             uint8_t* __restrict__ q, float* __restrict__ s,
                                                             int early) {
  if (early) pdl_launch();
  pdl_wait();
  constexpr float kQmax = INT8 ? 127.0f : 448.0f;
  constexpr int W = sizeof(T) / 2;  // 16-byte words of 8 values
  constexpr int NV = 128 / LPG;     // values a lane
  constexpr int NC = NV / 8;        // 8-value chunks a lane
  constexpr int GPS = 32 / LPG;     // groups a warp step
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPG, l = lane % LPG;  // the group within the warp step, the lane within the group
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t p = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * U; GPS * p < groups;
       p += warps * U) {
    uint4 w[U][NC][W];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = GPS * (p + u) + sub;
#pragma unroll
      for (int h = 0; h < NC; ++h) {
        if (g < groups) {
          raw_load8(x + g * 128 + l * NV + h * 8, w[u][h]);
        } else {
#pragma unroll
          for (int i = 0; i < W; ++i) w[u][h][i] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = GPS * (p + u) + sub;
      float v[NC][8];
#pragma unroll
      for (int h = 0; h < NC; ++h) unpack8(w[u][h], x, v[h]);
      float amax = 0.0f;
#pragma unroll
      for (int h = 0; h < NC; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[h][i]));
#pragma unroll
      for (int o = LPG / 2; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), kQmax);
#pragma unroll
      for (int h = 0; h < NC; h += 2) {
        const uint2 c0 = block_codes8<INT8>(v[h], sc);
        const uint2 c1 = block_codes8<INT8>(v[h + 1], sc);
        if (g < groups) *reinterpret_cast<uint4*>(q + g * 128 + l * NV + h * 8) = make_uint4(c0.x, c0.y, c1.x, c1.y);
      }
      if (g < groups && l == 0) s[g] = sc;
    }
  }
  if (!early) pdl_launch();
}

// ---------------------------------------------------------------------------------------------------------------
// Weights, FP8 / INT8 block formats: one CTA per 128 x 128 block (basal/blockquant.py:126-135).
// ---------------------------------------------------------------------------------------------------------------
template <typename T, bool INT8>
__global__ void __launch_bounds__(256) weight_quant_block_kernel(const T* __restrict__ w, int64_t K,
                                                                 uint8_t* __restrict__ q, float* __restrict__ s) {
  constexpr float kQmax = INT8 ? 127.0f : 448.0f;
  __shared__ float red[8];
  const int kb = blockIdx.x, nb = blockIdx.y, t = threadIdx.x;
  const int r = t >> 1, c0 = (t & 1) * 64;
  const int64_t base = ((int64_t)nb * 128 + r) * K + (int64_t)kb * 128 + c0;
  float amax = 0.0f;
#pragma unroll
  for (int c = 0; c < 64; c += 8) {
    float v[8];
    load8(w + base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), kQmax);
#pragma unroll
  for (int c = 0; c < 64; c += 8) {
    float v[8];
    load8(w + base + c, v);
    *reinterpret_cast<uint2*>(q + base + c) = block_codes8<INT8>(v, sc);
  }
  if (t == 0) s[(int64_t)nb * gridDim.x + kb] = sc;
}

// ---------------------------------------------------------------------------------------------------------------
// NVFP4
// ---------------------------------------------------------------------------------------------------------------
// e2m1 code of u (in units of the block scale): the cuts of basal/nvfp4.py:22 (ties to the even code), sign bit 3
// for every u < 0 (nvfp4.py:36-41).
__device__ __forceinline__ uint32_t e2m1_code(float u) {
  const float a = fabsf(u);
  uint32_t c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
  return c | ((u < 0.0f) ? 8u : 0u);
}

// 8 quotients -> 8 e2m1 codes, the first in the low nibble: the hardware conversion rounds to nearest even and
// saturates at 6, which is the reference's CUTS (a > 0.25, a >= 0.75, a > 1.25, a >= 1.75, a > 2.5, a >= 3.5, a > 5).
// The one difference, -0 (code 8 from the hardware, 0 from the reference), the caller removes: no quotient may be -0.
__device__ __forceinline__ uint32_t e2m1_codes8(const float (&z)[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(z[0]), "f"(z[1]), "f"(z[2]), "f"(z[3]), "f"(z[4]), "f"(z[5]), "f"(z[6]), "f"(z[7]));
  return out;
}

// Distance, in units of y's last place, from y to the nearest value whose low 21 mantissa bits are zero (wrapped:
// small means near). y = RN(v * RN(1 / sc)) is within 2 ulp of the exact quotient v / sc, and every e2m1 code
// threshold (0.25 ... 5) is such a value, so y and the correctly rounded quotient give the same code when the
// distance is above 16 (8 ulp). A zero y also lands at or below 16, so a zero or an underflowed product takes the
// exact division too, which keeps the sign rule of the reference's quotient.
__device__ __forceinline__ uint32_t e2m1_cut_distance(float y) { return (__float_as_uint(y) + 8u) & 0x1FFFFFu; }

__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float v = mag[c & 7];
  return (c & 8) ? -v : v;
}

// Byte offset of scale (row r, 16-group j) in the 128 x 4 tile swizzle of a matrix with `c4` tiles a row
// (basal/nvfp4.py:49-56, :140-143).
__device__ __forceinline__ int64_t swizzled_scale_offset(int64_t r, int64_t j, int64_t c4) {
  return ((r >> 7) * c4 + (j >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (j & 3);
}

// One CTA per 128 rows x TILES tiles of 64 features, one thread per (row, 16-group) of each tile: all the thread's
// loads first, then per tile the codes and the tile's 512 scale bytes, staged in shared memory and written as 16-byte
// stores. Rows past M (up to the 128-row padding) get zeros. TILES = 2 when there are enough tiles to fill the GPU
// (0.42 of HBM at 8192 x 6144 bf16, against 0.35 with 1 tile and 0.30 with 4), else 1.
template <typename T, int TILES>
__global__ void __launch_bounds__(512) nvfp4_act_quant_kernel(const T* __restrict__ x, const float* __restrict__ inv_g_p,
                                                              int64_t M, int64_t K, uint8_t* __restrict__ q,
                                                              uint8_t* __restrict__ s, int early) {
  if (early) pdl_launch();  // as in act_quant_block_kernel
  pdl_wait();
  constexpr int W = sizeof(T) / 2;  // 16-byte words of 8 values
  __shared__ __align__(16) uint8_t sbuf[TILES][512];
  const int64_t tile_r = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * TILES;  // first 64-feature tile
  const int nt = (int)(K / 64 - c0 < TILES ? K / 64 - c0 : TILES);
  const int t = threadIdx.x;
  const int r = t >> 2, j = t & 3;
  const int64_t row = tile_r * 128 + r;
  const bool live = row < M;
  uint4 w[TILES][2][W];
#pragma unroll
  for (int c = 0; c < TILES; ++c) {
    if (c < nt && live) {
      const T* p = x + row * K + (c0 + c) * 64 + j * 16;
      raw_load8(p, w[c][0]);
      raw_load8(p + 8, w[c][1]);
    }
  }
  const float inv_g = __ldg(inv_g_p);
#pragma unroll
  for (int c = 0; c < TILES; ++c) {
    if (c >= nt) break;
    uint32_t scale_bits = 0, lo = 0, hi = 0;
    if (live) {
      float v[16];
      unpack8(w[c][0], x, *reinterpret_cast<float(*)[8]>(v));
      unpack8(w[c][1], x, *reinterpret_cast<float(*)[8]>(v + 8));
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = __fmul_rn(v[i], inv_g);
        amax = fmaxf(amax, fabsf(v[i]));
      }
      const uint8_t sb = float_to_e4m3(fminf(__fdiv_rn(amax, 6.0f), 448.0f));
      const float sf = e4m3_to_float(sb);
      scale_bits = sb;
      // u = v / sf as an IEEE division (nvfp4.py:106-112), 0 where sf is 0: RN(v * RN(1 / sf) + 0) (the + 0 turns
      // a -0 into +0, the reference's code 0) unless a product lies near a code threshold or is 0, then the group
      // takes the division
      float u[16];
      if (sf > 0.0f) {
        const float rcp = __frcp_rn(sf);
        uint32_t dmin = 0xFFFFFFFFu;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          u[i] = __fmaf_rn(v[i], rcp, 0.0f);
          dmin = min(dmin, e2m1_cut_distance(u[i]));
        }
        if (dmin <= 16u) {
#pragma unroll
          for (int i = 0; i < 16; ++i) u[i] = __fadd_rn(__fdiv_rn(v[i], sf), 0.0f);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) u[i] = 0.0f;
      }
      lo = e2m1_codes8(*reinterpret_cast<const float(*)[8]>(u));
      hi = e2m1_codes8(*reinterpret_cast<const float(*)[8]>(u + 8));
    }
    *reinterpret_cast<uint2*>(q + row * (K / 2) + (c0 + c) * 32 + j * 8) = make_uint2(lo, hi);
    sbuf[c][(r & 31) * 16 + (r >> 5) * 4 + j] = static_cast<uint8_t>(scale_bits);
  }
  __syncthreads();
  if (t < 32 * nt) {
    const int c = t >> 5;
    const int64_t tile = tile_r * (K / 64) + c0 + c;
    reinterpret_cast<uint4*>(s + tile * 512)[t & 31] = reinterpret_cast<const uint4*>(sbuf[c])[t & 31];
  }
  if (!early) pdl_launch();
}

// ---- NVFP4 weights (basal/nvfp4.py:75-97) ----
// Largest |w| into g[0] (as fp32 bits; g zeroed before): the weights' global amax.
template <typename T>
__global__ void __launch_bounds__(256) absmax_kernel(const T* __restrict__ w, int64_t n8, unsigned* __restrict__ out) {
  float amax = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    load8(w + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(amax));
}

// One thread per 16-block of the weight's scale tiles: Np = N rounded up to 128 rows, c4 tiles of 4 blocks a row
// (K / 16 blocks rounded up to 4); blocks past N rows or past K / 16 columns get a zero scale (the padding of
// basal/nvfp4.py:49-56).
// g = max(amax / (6 * 448), 1e-12); b = w / g; per candidate f: s = e4m3(min(amax16 * f / 6, 448)), codes of b / s,
// squared error summed as torch's CPU kernel sums 16 values (lanes k and k + 8, then 0 + p0 + ... + p7); the
// smallest error wins, the earlier candidate on a tie.
template <typename T>
__global__ void __launch_bounds__(256) nvfp4_weight_quant_kernel(const T* __restrict__ w, const float* __restrict__ gbuf,
                                                                 int64_t N, int64_t Np, int64_t K, int64_t c4,
                                                                 uint8_t* __restrict__ codes,
                                                                 uint8_t* __restrict__ scales) {
  const int64_t kb16 = K / 16, cols = c4 * 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= Np * cols) return;
  const int64_t row = idx / cols, j = idx - row * cols;
  if (row >= N || j >= kb16) {
    scales[swizzled_scale_offset(row, j, c4)] = 0;
    return;
  }
  const float g = fmaxf(__fdiv_rn(__ldg(gbuf), 2688.0f), 1e-12f);
  float b[16];
  {
    float a[8], c[8];
    load8(w + row * K + j * 16, a);
    load8(w + row * K + j * 16 + 8, c);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      b[i] = a[i];
      b[8 + i] = c[i];
    }
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    b[i] = __fdiv_rn(b[i], g);
    amax = fmaxf(amax, fabsf(b[i]));
  }
  // the candidates 1 - 0.04 j, computed in double by the reference and rounded to fp32 where they meet amax
  const float cand[8] = {(float)(1.0 - 0.04 * 0), (float)(1.0 - 0.04 * 1), (float)(1.0 - 0.04 * 2),
                         (float)(1.0 - 0.04 * 3), (float)(1.0 - 0.04 * 4), (float)(1.0 - 0.04 * 5),
                         (float)(1.0 - 0.04 * 6), (float)(1.0 - 0.04 * 7)};
  float best_err = 0.0f;
  uint32_t best_lo = 0, best_hi = 0, best_s = 0;
#pragma unroll 1
  for (int f = 0; f < 8; ++f) {
    const uint8_t sb = float_to_e4m3(fminf(__fdiv_rn(__fmul_rn(amax, cand[f]), 6.0f), 448.0f));
    const float sf = e4m3_to_float(sb);
    uint32_t lo = 0, hi = 0;
    float d[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float u = sf > 0.0f ? __fdiv_rn(b[i], sf) : 0.0f;
      const uint32_t c = e2m1_code(u);
      if (i < 8)
        lo |= c << (4 * i);
      else
        hi |= c << (4 * (i - 8));
      const float e = __fsub_rn(__fmul_rn(e2m1_value(c), sf), b[i]);
      d[i] = __fmul_rn(e, e);
    }
    float err = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) err = __fadd_rn(err, __fadd_rn(d[k], d[k + 8]));
    if (f == 0 || err < best_err) {
      best_err = err;
      best_lo = lo;
      best_hi = hi;
      best_s = sb;
    }
  }
  *reinterpret_cast<uint2*>(codes + row * (K / 2) + j * 8) = make_uint2(best_lo, best_hi);
  scales[swizzled_scale_offset(row, j, c4)] = static_cast<uint8_t>(best_s);
}

__global__ void nvfp4_global_scale_kernel(float* g) {
  g[0] = fmaxf(__fdiv_rn(g[0], 2688.0f), 1e-12f);
}

}  // namespace b200
