// The config-5 hybrid decoder's element-wise steps around its FP8-block linears, each one kernel that reads the
// previous step's output once and writes the next GEMM's operand (the maths of the reference's Qwen 3.5 graph forward,
// basal/gdn_graph.py:122-140, :432-439, with the roundings of its torch ops):
//
//   rms_quant_kernel      Qwen3_5RMSNorm (1 + w) of a row, rounded to 16 bits, quantised into 1 x 128 e4m3 groups:
//                         the A operand (codes, scales) of the next block GEMM, and optionally the normed row itself
//   gdn_prep_kernel       the Gated DeltaNet's causal depthwise convolution (k taps) + SiLU over the q / k / v
//                         channels of the merged input projection, rounded to 16 bits, the l2 norms of q and k (q also
//                         scaled by dk^-1/2), beta = sigmoid(b), g = -e^A_log softplus(a + dt_bias): the recurrence's
//                         operands, head-major: q, k [rows, key heads, T, d] fp32, v [rows, value heads, T, d] in
//                         the 16-bit type (its values are 16-bit already), beta, g [rows, value heads, T] fp32
//   gdn_gate_quant_kernel the Gated DeltaNet's output: each value head's 128 values rounded to 16 bits, RMS-normed,
//                         times the norm weight, times SiLU(z), rounded, and quantised as one 1 x 128 group (a head is
//                         exactly one group of the output projection's input)
//
// Every multiply and add that torch rounds on its own is __fmul_rn / __fadd_rn (no contraction into an FMA);
// exponentials and divisions are expf / __fdiv_rn, as torch's CUDA kernels compute silu, sigmoid and softplus. The
// sums of squares of the norms are fp32 in this kernel's own order (torch's reduction order is not part of the
// contract), so a normed value may differ from torch's by one unit in the last place.
#pragma once
#include "quant.cuh"

namespace b200 {
namespace hybrid {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }

// v rounded to T and back (the value a torch op on T tensors leaves)
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f<T>(from_f<T>(v));
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// 8 16-bit values -> fp32
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]) {
  uint4 w[1];
  raw_load8(p, w);
  unpack8(w, p, v);
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ---------------------------------------------------------------------------------------------------------------
// RMSNorm + FP8 quantiser: a warp per row of D features (D % 128 == 0). Pass 1 sums the squares (lane l holds the
// 8-value chunks l, l + 32, ...: 256 consecutive features a warp step, as the quantiser's half-warp groups), pass 2
// reloads the row (L1 / L2), forms y = RN16(RN(x * r) * RN(1 + w)) with r = rsqrt(mean + eps), and quantises each
// 128-feature group exactly as act_quant_block_kernel does (half-warp amax, scale = RN(max(amax, 1e-12) / 448),
// block_codes8), so the codes equal the standalone quantiser's of y.
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rms_quant_kernel(const T* __restrict__ x, const T* __restrict__ w, float eps,
                                                        int64_t M, int D, T* __restrict__ y,
                                                        uint8_t* __restrict__ q, float* __restrict__ s) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row < M) {
    const T* xr = x + row * D;
    float ss = 0.0f;
    for (int c = lane * 8; c < D; c += 256) {
      float v[8];
      ld8(xr + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    const int groups = D / 128;
    for (int base = 0; base < D; base += 256) {
      const int c = base + lane * 8;
      const bool live = c < D;  // the last step of a D % 256 == 128 row: its upper half-warp has no group
      float v[8];
      if (live) {
        float xv[8], wv[8];
        ld8(xr + c, xv);
        ld8(w + c, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = round_to<T>(__fmul_rn(__fmul_rn(xv[i], r), __fadd_rn(1.0f, wv[i])));
        if (y) st8(y + row * D + c, v);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
      }
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
      const uint2 codes = block_codes8<false>(v, sc);
      if (live) {
        *reinterpret_cast<uint2*>(q + row * D + c) = codes;
        if ((lane & 15) == 0) s[row * groups + c / 128] = sc;
      }
    }
  }
  pdl_launch();
}

// ---------------------------------------------------------------------------------------------------------------
// Gated DeltaNet input: a warp per (row r, token t, key head h); lane l owns channels 4l .. 4l + 3 of a 128-channel
// head. proj [rows * T, ld] holds, per token, the convolution's input channels [q (Hk * 128) | k (Hk * 128) | v (Hv *
// 128)] from column 0, then b at column b_off and a at a_off (one per value head). tail [tr, 3, C] (tr = 1: every
// row continues the same inputs; tr = rows; null: zeros) holds the 3 inputs before token 0, oldest first (4 taps).
// Convolution of channel c at token t: acc = x[t - 3] w[c, 0], then acc = RN(acc + RN(x[t - 3 + j] w[c, j])) for
// j = 1 .. 3 (torch's order in the unfused form: a product, then a sum, each rounded); y = RN16(silu(acc)). A lane
// reads its 4 channels of a tap as one 8-byte load and their 16 weights as two 16-byte loads.
// ---------------------------------------------------------------------------------------------------------------
struct PrepParams {
  const void* proj;
  int64_t ld;         // elements between tokens in proj
  const void* tail;   // [tr, 3, C] or null
  int tail_rows;      // 1 or rows
  const void* conv;   // [C, 4] 16-bit
  const float* A_log; // [Hv]
  const void* dt_bias;// [Hv] 16-bit
  int b_off, a_off;   // columns of b and a in proj
  int rows, T, Hk, Hv;
  float q_scale;      // dk^-1/2
  float* q;           // [rows, Hk, T, 128]
  float* k;
  void* v;            // [rows, Hv, T, 128] 16-bit
  float* beta;        // [rows, Hv, T]
  float* g;
};

// 4 consecutive 16-bit values (8 bytes) -> fp32
template <typename T>
__device__ __forceinline__ void ld4(const T* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = to_f<T>(h[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// A warp takes PTB consecutive tokens of one row and key head: the convolution window (PTB + 3 input rows) and the
// weights of each channel group are loaded once for the PTB tokens.
constexpr int PTB = 4;

// The convolution (4 taps) + SiLU of channels col .. col + 3 at tokens t0 .. t0 + PTB - 1 (those below ntok) from the
// window's rows src[w] (input token t0 - 3 + w; null: zeros): acc = x_0 w_0, then acc = RN(acc + RN(x_j w_j)) over
// the taps in order (torch's unfused products and sums); y = RN16(silu(acc)).
template <typename T>
__device__ __forceinline__ void conv4_tokens(const T* const (&src)[PTB + 3], const T* conv, int col,
                                             float (&y)[PTB][4]) {
  float w[16];  // channel i, tap j at w[4 i + j]: the 4 channels' weights are 32 contiguous bytes
  {
    const uint4 a = *reinterpret_cast<const uint4*>(conv + (int64_t)col * 4);
    const uint4 b = *reinterpret_cast<const uint4*>(conv + (int64_t)col * 4 + 8);
    const T* ha = reinterpret_cast<const T*>(&a);
    const T* hb = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[i] = to_f<T>(ha[i]);
      w[8 + i] = to_f<T>(hb[i]);
    }
  }
  float x[PTB + 3][4];
#pragma unroll
  for (int k = 0; k < PTB + 3; ++k) {
    x[k][0] = x[k][1] = x[k][2] = x[k][3] = 0.0f;
    if (src[k]) ld4(src[k] + col, x[k]);
  }
#pragma unroll
  for (int t = 0; t < PTB; ++t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float acc = __fmul_rn(x[t][i], w[4 * i]);
#pragma unroll
      for (int j = 1; j < 4; ++j) acc = __fadd_rn(acc, __fmul_rn(x[t + j][i], w[4 * i + j]));
      y[t][i] = round_to<T>(silu_f(acc));
    }
  }
}

// 3 CTAs an SM (80 registers, a few spilled): 0.661 -> 0.545 ms at a C5 micro-batch against 2 CTAs at 91 registers
template <typename T>
__global__ void __launch_bounds__(256, 3) gdn_prep_kernel(const PrepParams p) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nb = (p.T + PTB - 1) / PTB;
  if (item < (int64_t)p.rows * p.Hk * nb) {  // warp-uniform
    const int h = (int)(item % p.Hk);
    const int tb = (int)((item / p.Hk) % nb);
    const int r = (int)(item / ((int64_t)p.Hk * nb));
    const int t0 = tb * PTB, ntok = min(PTB, p.T - t0);
    const int C = (p.Hk * 2 + p.Hv) * 128;
    const T* proj = static_cast<const T*>(p.proj);
    const T* tail = static_cast<const T*>(p.tail);
    const T* conv = static_cast<const T*>(p.conv);
    const T* src[PTB + 3];  // input tokens t0 - 3 .. t0 + PTB - 1 (the tail's before token 0; null past the row)
#pragma unroll
    for (int k = 0; k < PTB + 3; ++k) {
      const int tt = t0 - 3 + k;
      if (tt >= p.T)
        src[k] = nullptr;
      else if (tt >= 0)
        src[k] = proj + ((int64_t)r * p.T + tt) * p.ld;
      else
        src[k] = tail ? tail + ((int64_t)(p.tail_rows == 1 ? 0 : r) * 3 + 3 + tt) * C : nullptr;
    }
    const int c0 = lane * 4;
    // q and k of key head h: l2 norms by warp sums (q also scaled), written once per key head
#pragma unroll
    for (int qk = 0; qk < 2; ++qk) {
      float y[PTB][4];
      conv4_tokens<T>(src, conv, qk * p.Hk * 128 + h * 128 + c0, y);
      float* out = qk == 0 ? p.q : p.k;
#pragma unroll
      for (int t = 0; t < PTB; ++t) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(y[t][i], y[t][i]));
        const float rn = rsqrtf(__fadd_rn(warp_sum(ss), 1e-6f));
        if (t < ntok) {
          float4 o4;
          if (qk == 0) {
            o4 = make_float4(__fmul_rn(__fmul_rn(y[t][0], rn), p.q_scale), __fmul_rn(__fmul_rn(y[t][1], rn), p.q_scale),
                             __fmul_rn(__fmul_rn(y[t][2], rn), p.q_scale), __fmul_rn(__fmul_rn(y[t][3], rn), p.q_scale));
          } else {
            o4 = make_float4(__fmul_rn(y[t][0], rn), __fmul_rn(y[t][1], rn), __fmul_rn(y[t][2], rn),
                             __fmul_rn(y[t][3], rn));
          }
          *reinterpret_cast<float4*>(out + (((int64_t)r * p.Hk + h) * p.T + t0 + t) * 128 + c0) = o4;
        }
      }
    }
    // v of the value heads of key head h, 16-bit (conv4 rounded them already)
    const int rep = p.Hv / p.Hk;
    for (int j = 0; j < rep; ++j) {
      const int vh = h * rep + j;
      float y[PTB][4];
      conv4_tokens<T>(src, conv, 2 * p.Hk * 128 + vh * 128 + c0, y);
#pragma unroll
      for (int t = 0; t < PTB; ++t) {
        if (t < ntok) {
          uint2 u;
          T* uh = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int i = 0; i < 4; ++i) uh[i] = from_f<T>(y[t][i]);
          *reinterpret_cast<uint2*>(static_cast<T*>(p.v) + (((int64_t)r * p.Hv + vh) * p.T + t0 + t) * 128 + c0) = u;
        }
      }
    }
    // beta and g: entry e = t * rep + j (lane e, e + 32, ..) for token t0 + t and value head h * rep + j
    for (int e = lane; e < ntok * rep; e += 32) {
      const int t = e / rep, vh = h * rep + e % rep;
      const T* pr = proj + ((int64_t)r * p.T + t0 + t) * p.ld;
      const float bb = to_f<T>(pr[p.b_off + vh]);
      const float aa = to_f<T>(pr[p.a_off + vh]);
      const int64_t bo = ((int64_t)r * p.Hv + vh) * p.T + t0 + t;
      p.beta[bo] = round_to<T>(sigmoid_f(bb));
      const float dt = to_f<T>(static_cast<const T*>(p.dt_bias)[vh]);
      p.g[bo] = __fmul_rn(-expf(p.A_log[vh]), softplus_f(__fadd_rn(aa, dt)));
    }
  }
  pdl_launch();
}

// ---------------------------------------------------------------------------------------------------------------
// Gated DeltaNet output + FP8 quantiser: a half-warp per (token, value head), 8 values a lane. o [rows, Hv, Tp, 128]
// (the recurrence's output, fp32 or already rounded to T; Tp >= ntok tokens a row), z in proj (16-bit, row stride ld,
// column z_off + vh * 128), gw [128]:
// u = RN16(o); n = RN16(RN(u * rsqrt(mean(u^2) + eps))); n = RN16(RN(gw * n)); out = RN16(RN(n * silu(z)));
// codes / scale of the 128 values as act_quant_block_kernel's, into q [rows * T, Hv * 128] / s [rows * T, Hv].
// ---------------------------------------------------------------------------------------------------------------
template <typename TO>
__device__ __forceinline__ void load_o8(const TO* p, float (&v)[8]) {
  uint4 w[sizeof(TO) / 2];
  raw_load8(p, w);
  unpack8(w, p, v);
}

template <typename T, typename TO>
__global__ void __launch_bounds__(256) gdn_gate_quant_kernel(const TO* __restrict__ o, int Tp,
                                                             const T* __restrict__ z, int64_t ld, int z_off,
                                                             const T* __restrict__ gw, float eps, int rows, int ntok,
                                                             int Hv, T* __restrict__ y, uint8_t* __restrict__ q,
                                                             float* __restrict__ s) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int l = lane & 15;
  const int64_t item = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + (lane >> 4);
  const int64_t items = (int64_t)rows * ntok * Hv;
  const bool live = item < items;
  float v[8];
  int64_t tok = 0;
  int vh = 0;
  if (live) {
    vh = (int)(item % Hv);
    tok = item / Hv;  // r * T + t
    const int t = (int)(tok % ntok), r = (int)(tok / ntok);
    load_o8(o + (((int64_t)r * Hv + vh) * Tp + t) * 128 + l * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = round_to<T>(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
#pragma unroll
  for (int o2 = 8; o2 >= 1; o2 >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o2));
  const float rr = rsqrtf(__fadd_rn(__fdiv_rn(ss, 128.0f), eps));
  if (live) {
    float zv[8], wv[8];
    ld8(z + tok * ld + z_off + vh * 128 + l * 8, zv);
    ld8(gw + l * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float n = round_to<T>(__fmul_rn(wv[i], round_to<T>(__fmul_rn(v[i], rr))));
      v[i] = round_to<T>(__fmul_rn(n, silu_f(zv[i])));
    }
    if (y) st8(y + tok * (int64_t)Hv * 128 + vh * 128 + l * 8, v);
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o2 = 8; o2 >= 1; o2 >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o2));
  const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  const uint2 codes = block_codes8<false>(v, sc);
  if (live) {
    *reinterpret_cast<uint2*>(q + tok * (int64_t)Hv * 128 + vh * 128 + l * 8) = codes;
    if (l == 0) s[tok * Hv + vh] = sc;
  }
  pdl_launch();
}

// ---------------------------------------------------------------------------------------------------------------
// Attention input: a warp per (token, head) of the merged q+gate / k / v projection (qkv [rows * T, ld], per token
// [H heads x (128 q, 128 gate) | Hk x 128 k | Hk x 128 v]), 4 values a lane. q and k heads: Qwen3_5RMSNorm with their
// weight (RN16(RN(x * r) * RN(1 + w)), r = rsqrt(mean(x^2) + eps)), then the rotary embedding of the first `rot`
// dimensions (x1 cos - x2 sin, x2 cos + x1 sin, every product and sum rounded to 16 bits as torch's ops round them;
// cos / sin [rows or 1, T, rot]); the partner dimensions rot / 2 away sit rot / 8 lanes away. q goes to q_out
// [rows, H, T, 128]; k and the head's v to k_out / v_out [rows, Hk, kv_len, 128] at position kv_off + t, so that the
// rows' keys land after a prefix's already in the buffer.
// ---------------------------------------------------------------------------------------------------------------
struct AttnPrepParams {
  const void* qkv;
  int64_t ld;
  int rows, T, H, Hk;
  const void* q_norm;   // [128]
  const void* k_norm;   // [128]
  float eps;
  const void* cos;      // [rows or 1, T, rot] 16-bit
  const void* sin;
  int64_t cs_row;       // elements between rows of cos / sin (0: shared)
  int rot;              // rotated dimensions (a multiple of 8, at most 128)
  void* q_out;
  void* k_out;
  void* v_out;
  int64_t kv_len, kv_off;
};

template <typename T>
__global__ void __launch_bounds__(256) attn_prep_kernel(const AttnPrepParams p) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int heads = p.H + p.Hk;
  if (item < (int64_t)p.rows * p.T * heads) {  // warp-uniform
    const int j = (int)(item % heads);
    const int64_t tok = item / heads;  // r * T + t
    const int t = (int)(tok % p.T), r = (int)(tok / p.T);
    const bool isq = j < p.H;
    const int h = isq ? j : j - p.H;
    const T* x = static_cast<const T*>(p.qkv) + tok * p.ld;
    const T* src = isq ? x + h * 256 : x + (int64_t)p.H * 256 + h * 128;
    const T* w = static_cast<const T*>(isq ? p.q_norm : p.k_norm);
    float v[4], wv[4];
    ld4(src + lane * 4, v);
    ld4(w + lane * 4, wv);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    const float rr = rsqrtf(__fadd_rn(__fdiv_rn(warp_sum(ss), 128.0f), p.eps));
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = round_to<T>(__fmul_rn(__fmul_rn(v[i], rr), __fadd_rn(1.0f, wv[i])));
    const int hl = p.rot / 8;  // lanes of half the rotated dimensions
    const int partner = lane < hl ? lane + hl : lane - hl;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float other = __shfl_sync(0xffffffffu, y[i], partner & 31);
      o[i] = y[i];
      if (lane < 2 * hl) {
        const int64_t ci = (int64_t)r * p.cs_row + (int64_t)t * p.rot + lane * 4 + i;
        const float c = to_f<T>(static_cast<const T*>(p.cos)[ci]);
        const float sn = to_f<T>(static_cast<const T*>(p.sin)[ci]);
        const float a = round_to<T>(__fmul_rn(y[i], c)), b = round_to<T>(__fmul_rn(other, sn));
        o[i] = lane < hl ? round_to<T>(__fsub_rn(a, b)) : round_to<T>(__fadd_rn(a, b));
      }
    }
    T* dst = isq ? static_cast<T*>(p.q_out) + (((int64_t)r * p.H + h) * p.T + t) * 128
                 : static_cast<T*>(p.k_out) + (((int64_t)r * p.Hk + h) * p.kv_len + p.kv_off + t) * 128;
    uint2 u;
    T* uh = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) uh[i] = from_f<T>(o[i]);
    *reinterpret_cast<uint2*>(dst + lane * 4) = u;
    if (!isq) {  // the head's values, copied
      const T* vs = x + (int64_t)p.H * 256 + (int64_t)p.Hk * 128 + h * 128 + lane * 4;
      T* vd = static_cast<T*>(p.v_out) + (((int64_t)r * p.Hk + h) * p.kv_len + p.kv_off + t) * 128 + lane * 4;
      *reinterpret_cast<uint2*>(vd) = *reinterpret_cast<const uint2*>(vs);
    }
  }
  pdl_launch();
}

// ---------------------------------------------------------------------------------------------------------------
// Attention output gate + FP8 quantiser: a half-warp per (token, head), 8 values a lane. o [rows, H, T, 128] (the
// attention's output), gate in qkv (the second 128 values of each head's q+gate pair): a = RN16(o * RN16(sigmoid(g)))
// as torch computes o * sigmoid(gate) in 16 bits; each head's 128 values are one quantisation group of the output
// projection's input: codes q [rows * T, H * 128], scales s [rows * T, H], as act_quant_block_kernel's.
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) attn_gate_quant_kernel(const T* __restrict__ o, const T* __restrict__ qkv,
                                                              int64_t ld, int rows, int ntok, int H,
                                                              uint8_t* __restrict__ q, float* __restrict__ s) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int l = lane & 15;
  const int64_t item = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 2 + (lane >> 4);
  const bool live = item < (int64_t)rows * ntok * H;
  float v[8];
  int64_t tok = 0;
  int h = 0;
  if (live) {
    h = (int)(item % H);
    tok = item / H;  // r * T + t
    const int t = (int)(tok % ntok), r = (int)(tok / ntok);
    float ov[8], gv[8];
    ld8(o + (((int64_t)r * H + h) * ntok + t) * 128 + l * 8, ov);
    ld8(qkv + tok * ld + h * 256 + 128 + l * 8, gv);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = round_to<T>(__fmul_rn(ov[i], round_to<T>(sigmoid_f(gv[i]))));
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o2 = 8; o2 >= 1; o2 >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o2));
  const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  const uint2 codes = block_codes8<false>(v, sc);
  if (live) {
    *reinterpret_cast<uint2*>(q + tok * (int64_t)H * 128 + h * 128 + l * 8) = codes;
    if (l == 0) s[tok * H + h] = sc;
  }
  pdl_launch();
}

}  // namespace hybrid
}  // namespace b200
