// The gated delta rule of the Gated DeltaNet layers (the recurrence of transformers' torch_chunk_gated_delta_rule /
// fla's chunk_gated_delta_rule, which the reference's Qwen 3.5 graph forward calls, basal/gdn_graph.py:81-87,
// :492-493), over chunks of 64 tokens, in fp32.
//
// Per value head, with l2-normed keys k_t, scaled queries q_t, values v_t, gates g_t <= 0 and beta_t in (0, 1), the
// state S [dk = 128, dv = 128] follows S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T and the
// output is o_t = S_t^T q_t. Over a chunk with cumulative gates G (G_i = g_1 + .. + g_i within the chunk):
//   A_ij = beta_i (k_i . k_j) e^{G_i - G_j} (j < i), T = (I + A)^-1 (unit lower triangular)
//   U = T (beta V),  W = T (beta e^G K),  V' = U - W S,
//   O = e^G (Q S) + (Q K^T (.) e^{G_i - G_j}, j <= i) V',  S <- e^{G_last} S + (e^{G_last - G} K)^T V'.
//
// A CTA owns one (row, value head) and one half of the value dimension (64 of S's 128 columns): the products that do
// not involve V (A, T, W, Q K^T) are computed by both halves. 256 threads; every product is a register-tiled fp32 FMA
// loop over shared memory with the left operand stored transposed ([k][rows]: a thread's rows are one float4) and the
// right one row-major ([k][cols]: a thread's columns are one or two float4), so every shared-memory read is a
// contiguous vector. T is found by 16 x 16 blocks: the diagonal blocks by forward substitution (a warp each), the
// off-diagonal ones by T_IJ = -T_II sum_{M = J .. I - 1} A_IM T_MJ, one block distance at a time.
#pragma once
#include "common.cuh"

namespace b200 {
namespace gdnchunk {

constexpr int CH = 64;    // tokens a chunk
constexpr int DK = 128;   // key dim
constexpr int DV = 128;   // value dim
constexpr int DH = 64;    // value columns a CTA owns
constexpr int NT = 256;   // threads

struct Params {
  const float* q;      // [rows, H, T, 128] (l2-normed, scaled)
  const float* k;      // [rows, H, T, 128] (l2-normed)
  const float* v;      // [rows, H, T, 128]
  const float* g;      // [rows, H, T]
  const float* beta;   // [rows, H, T]
  const float* s0;     // [s0_rows, H, 128, 128] or null (zeros); s0_rows 1 (shared) or rows
  int s0_rows;
  float* o;            // [rows, H, T, 128]
  float* s_out;        // [rows, H, 128, 128] or null
  int rows, H, T;
};

struct Smem {
  float S[DK * DH];    // the state's columns of this CTA, [kk][c]
  float K[CH * DK];    // keys, row-major [i][kk]
  float KT[DK * CH];   // keys transposed [kk][i]; after the products with K^T: W transposed [kk][i]
  float QT[DK * CH];   // queries transposed [kk][i]
  float V[CH * DH];    // beta V, then V' = U - W S ([i][c])
  float A[CH * CH];    // A row-major [i][j]
  float Tm[CH * CH];   // T row-major, then transposed [j][i]
  float PT[CH * CH];   // (Q K^T (.) decay, causal) transposed [j][i]
  float G[CH];         // cumulative gates
  float B[CH];         // beta
};

// acc[RT][CT] += sum_k AT[k][r0 + i] * B[k][c0 + j] (fp32 FMAs, k ascending); RT, CT multiples of 4.
template <int RT, int CT, int KN, int LDA, int LDB>
__device__ __forceinline__ void mm(const float* __restrict__ AT, const float* __restrict__ Bm, int r0, int c0,
                                   float (&acc)[RT][CT]) {
#pragma unroll 4
  for (int k = 0; k < KN; ++k) {
    float a[RT], b[CT];
#pragma unroll
    for (int i = 0; i < RT; i += 4) *reinterpret_cast<float4*>(&a[i]) = *reinterpret_cast<const float4*>(AT + k * LDA + r0 + i);
#pragma unroll
    for (int j = 0; j < CT; j += 4) *reinterpret_cast<float4*>(&b[j]) = *reinterpret_cast<const float4*>(Bm + k * LDB + c0 + j);
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int j = 0; j < CT; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
  }
}

template <int RT, int CT>
__device__ __forceinline__ void zero(float (&acc)[RT][CT]) {
#pragma unroll
  for (int i = 0; i < RT; ++i)
#pragma unroll
    for (int j = 0; j < CT; ++j) acc[i][j] = 0.0f;
}

// T = (I + A)^-1 for the strictly lower A [64][64] (row-major in sh.A) -> sh.Tm row-major.
__device__ __forceinline__ void unit_lower_inverse(Smem& sh, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  // diagonal 16 x 16 blocks: warp b, lane j < 16 owns column j of block b; rows in order
  if (warp < 4) {
    const int b0 = warp * 16;
    float* T = sh.Tm;
    const float* A = sh.A;
    if (lane < 16)
      for (int i = 0; i < 16; ++i) T[(b0 + i) * CH + b0 + lane] = (i == lane) ? 1.0f : 0.0f;
    __syncwarp();
    for (int i = 1; i < 16; ++i) {
      float acc = 0.0f;
      if (lane < i) {
        for (int m = lane; m < i; ++m) acc = fmaf(A[(b0 + i) * CH + b0 + m], T[(b0 + m) * CH + b0 + lane], acc);
      }
      __syncwarp();
      if (lane < i) T[(b0 + i) * CH + b0 + lane] = -acc;
      __syncwarp();
    }
  }
  // the blocks above the diagonal are zero
  for (int e = tid; e < CH * CH; e += NT) {
    const int i = e / CH, j = e % CH;
    if ((j >> 4) > (i >> 4)) sh.Tm[e] = 0.0f;
  }
  __syncthreads();
  // off-diagonal blocks, distance d = I - J: a warp per block, lane owns 8 of its 256 entries (row lane / 2, columns
  // (lane % 2) * 8 ..)
  for (int d = 1; d < 4; ++d) {
    float x[8];
    const int blk = warp;  // block J = blk, I = blk + d
    const bool on = blk + d < 4;
    const int I0 = (blk + d) * 16, J0 = blk * 16;
    const int r = lane >> 1, cb = (lane & 1) * 8;
    if (on) {
#pragma unroll
      for (int c = 0; c < 8; ++c) x[c] = 0.0f;
      // X = sum_{M = J .. I - 1} A_IM T_MJ
      for (int m = J0; m < I0; ++m) {
        const float a = sh.A[(I0 + r) * CH + m];
#pragma unroll
        for (int c = 0; c < 8; ++c) x[c] = fmaf(a, sh.Tm[m * CH + J0 + cb + c], x[c]);
      }
    }
    __syncthreads();  // every warp has read the blocks it needs before any block of distance d is written
    // T_IJ = -T_II X: stage X in the (I, J) block of PT (free until the products with Q K^T)
    if (on) {
#pragma unroll
      for (int c = 0; c < 8; ++c) sh.PT[(I0 + r) * CH + J0 + cb + c] = x[c];
    }
    __syncthreads();
    if (on) {
      float y[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) y[c] = 0.0f;
      for (int m = 0; m < 16; ++m) {
        const float t = sh.Tm[(I0 + r) * CH + I0 + m];
#pragma unroll
        for (int c = 0; c < 8; ++c) y[c] = fmaf(t, sh.PT[(I0 + m) * CH + J0 + cb + c], y[c]);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) sh.Tm[(I0 + r) * CH + J0 + cb + c] = -y[c];
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NT, 1) gdn_chunk_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sh = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int half = blockIdx.x & 1;
  const int rh = blockIdx.x >> 1;  // r * H + h
  const int r = rh / p.H, h = rh % p.H;
  const int64_t base = (int64_t)rh * p.T;  // token row of (r, h, t = 0) in q / k / v / o, and in g / beta
  pdl_wait();
  // the initial state's columns of this half
  for (int e = tid * 4; e < DK * DH; e += NT * 4) {
    const int kk = e / DH, c = e % DH;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.s0) {
      const int sr = p.s0_rows == 1 ? 0 : r;
      s = *reinterpret_cast<const float4*>(p.s0 + (((int64_t)sr * p.H + h) * DK + kk) * DV + half * DH + c);
    }
    *reinterpret_cast<float4*>(&sh.S[e]) = s;
  }
  const int rb = tid >> 4, cb = tid & 15;
  for (int t0 = 0; t0 < p.T; t0 += CH) {
    const int n = min(CH, p.T - t0);
    // ---- chunk loads: K row-major (float4 along kk), K and Q transposed (a lane per token), beta V, G, beta ----
    for (int e = tid; e < CH * DK / 4; e += NT) {
      const int i = e / (DK / 4), f = e % (DK / 4);
      float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n) val = __ldg(reinterpret_cast<const float4*>(p.k + (base + t0 + i) * DK) + f);
      *reinterpret_cast<float4*>(&sh.K[i * DK + 4 * f]) = val;
    }
    for (int e = tid; e < CH * DK / 4; e += NT) {
      const int i = e % CH, f = e / CH;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), qv = kv;
      if (i < n) {
        kv = __ldg(reinterpret_cast<const float4*>(p.k + (base + t0 + i) * DK) + f);
        qv = __ldg(reinterpret_cast<const float4*>(p.q + (base + t0 + i) * DK) + f);
      }
      sh.KT[(4 * f + 0) * CH + i] = kv.x;
      sh.KT[(4 * f + 1) * CH + i] = kv.y;
      sh.KT[(4 * f + 2) * CH + i] = kv.z;
      sh.KT[(4 * f + 3) * CH + i] = kv.w;
      sh.QT[(4 * f + 0) * CH + i] = qv.x;
      sh.QT[(4 * f + 1) * CH + i] = qv.y;
      sh.QT[(4 * f + 2) * CH + i] = qv.z;
      sh.QT[(4 * f + 3) * CH + i] = qv.w;
    }
    if (tid < CH) {
      sh.B[tid] = tid < n ? __ldg(p.beta + base + t0 + tid) : 0.0f;
      sh.G[tid] = tid < n ? __ldg(p.g + base + t0 + tid) : 0.0f;
    }
    __syncthreads();
    if (tid == 0) {  // cumulative gates, in token order
      float acc = 0.0f;
      for (int i = 0; i < CH; ++i) {
        acc += sh.G[i];
        sh.G[i] = acc;
      }
    }
    for (int e = tid; e < CH * DH / 4; e += NT) {  // beta V
      const int i = e / (DH / 4), f = e % (DH / 4);
      float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n) {
        val = __ldg(reinterpret_cast<const float4*>(p.v + (base + t0 + i) * DV + half * DH) + f);
        const float bt = sh.B[i];
        val.x *= bt;
        val.y *= bt;
        val.z *= bt;
        val.w *= bt;
      }
      *reinterpret_cast<float4*>(&sh.V[i * DH + 4 * f]) = val;
    }
    __syncthreads();
    // ---- A = beta_i (k_i . k_j) e^{G_i - G_j} (j < i); P = (q_i . k_j) e^{G_i - G_j} (j <= i), stored transposed ----
    {
      float kk[4][4], qk[4][4];
      zero(kk);
      zero(qk);
      mm<4, 4, DK, CH, CH>(sh.KT, sh.KT, rb * 4, cb * 4, kk);
      mm<4, 4, DK, CH, CH>(sh.QT, sh.KT, rb * 4, cb * 4, qk);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int i = rb * 4 + a;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int j = cb * 4 + b;
          const float dec = j <= i ? expf(sh.G[i] - sh.G[j]) : 0.0f;
          sh.A[i * CH + j] = j < i ? sh.B[i] * kk[a][b] * dec : 0.0f;
          sh.PT[j * CH + i] = qk[a][b] * dec;
        }
      }
    }
    __syncthreads();
    // ---- T = (I + A)^-1 (uses PT's blocks below the diagonal as scratch, so P is stored again after) ----
    {
      float save[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) save[a][b] = sh.PT[(rb * 4 + a) * CH + cb * 4 + b];
      __syncthreads();
      unit_lower_inverse(sh, tid);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sh.PT[(rb * 4 + a) * CH + cb * 4 + b] = save[a][b];
      // T transposed in place (each thread its 4 x 4 block's entries, through registers)
      float t[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) t[a][b] = sh.Tm[(rb * 4 + a) * CH + cb * 4 + b];
      __syncthreads();
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sh.Tm[(cb * 4 + b) * CH + rb * 4 + a] = t[a][b];
    }
    __syncthreads();
    // ---- U = T (beta V) [64 x 64] and W = T (beta e^G K) [64 x 128] (W stored transposed over KT) ----
    float u[4][4];
    zero(u);
    mm<4, 4, CH, CH, DH>(sh.Tm, sh.V, rb * 4, cb * 4, u);
    {
      float w[4][8];
      zero(w);
#pragma unroll 2
      for (int k = 0; k < CH; ++k) {
        const float sc = sh.B[k] * expf(sh.G[k]);
        float a[4], b[8];
        *reinterpret_cast<float4*>(&a[0]) = *reinterpret_cast<const float4*>(sh.Tm + k * CH + rb * 4);
        *reinterpret_cast<float4*>(&b[0]) = *reinterpret_cast<const float4*>(sh.K + k * DK + cb * 8);
        *reinterpret_cast<float4*>(&b[4]) = *reinterpret_cast<const float4*>(sh.K + k * DK + cb * 8 + 4);
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] *= sc;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) w[i][j] = fmaf(a[i], b[j], w[i][j]);
      }
      __syncthreads();  // KT's last readers (the products above) are done
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sh.KT[(cb * 8 + j) * CH + rb * 4 + i] = w[i][j];
    }
    __syncthreads();
    // ---- V' = U - W S [64 x 64] (into V) ----
    {
      float ws[4][4];
      zero(ws);
      mm<4, 4, DK, CH, DH>(sh.KT, sh.S, rb * 4, cb * 4, ws);
      __syncthreads();  // every thread has read beta V
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        float4 vv;
        vv.x = u[a][0] - ws[a][0];
        vv.y = u[a][1] - ws[a][1];
        vv.z = u[a][2] - ws[a][2];
        vv.w = u[a][3] - ws[a][3];
        *reinterpret_cast<float4*>(&sh.V[(rb * 4 + a) * DH + cb * 4]) = vv;
      }
    }
    __syncthreads();
    // ---- O = e^G (Q S) + P V' ----
    {
      float o[4][4], pv[4][4];
      zero(o);
      zero(pv);
      mm<4, 4, DK, CH, DH>(sh.QT, sh.S, rb * 4, cb * 4, o);
      mm<4, 4, CH, CH, DH>(sh.PT, sh.V, rb * 4, cb * 4, pv);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int i = rb * 4 + a;
        if (i < n) {
          const float eg = expf(sh.G[i]);
          float4 ov;
          ov.x = fmaf(eg, o[a][0], pv[a][0]);
          ov.y = fmaf(eg, o[a][1], pv[a][1]);
          ov.z = fmaf(eg, o[a][2], pv[a][2]);
          ov.w = fmaf(eg, o[a][3], pv[a][3]);
          *reinterpret_cast<float4*>(p.o + (base + t0 + i) * DV + half * DH + cb * 4) = ov;
        }
      }
    }
    // ---- S <- e^{G_last} S + (e^{G_last - G} K)^T V' [128 x 64] ----
    {
      const float gl = sh.G[CH - 1];
      float sn[8][4];
      zero(sn);
#pragma unroll 2
      for (int k = 0; k < CH; ++k) {
        const float sc = expf(gl - sh.G[k]);
        float a[8], b[4];
        *reinterpret_cast<float4*>(&a[0]) = *reinterpret_cast<const float4*>(sh.K + k * DK + rb * 8);
        *reinterpret_cast<float4*>(&a[4]) = *reinterpret_cast<const float4*>(sh.K + k * DK + rb * 8 + 4);
        *reinterpret_cast<float4*>(&b[0]) = *reinterpret_cast<const float4*>(sh.V + k * DH + cb * 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] *= sc;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) sn[i][j] = fmaf(a[i], b[j], sn[i][j]);
      }
      const float egl = expf(gl);
      float old[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) old[i][j] = sh.S[(rb * 8 + i) * DH + cb * 4 + j];
      __syncthreads();  // every thread has read S (Q S, W S) and its entries of it
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sh.S[(rb * 8 + i) * DH + cb * 4 + j] = fmaf(egl, old[i][j], sn[i][j]);
    }
    __syncthreads();
  }
  if (p.s_out) {
    for (int e = tid * 4; e < DK * DH; e += NT * 4) {
      const int kk = e / DH, c = e % DH;
      *reinterpret_cast<float4*>(p.s_out + ((int64_t)rh * DK + kk) * DV + half * DH + c) =
          *reinterpret_cast<const float4*>(&sh.S[e]);
    }
  }
  pdl_launch();
}

}  // namespace gdnchunk
}  // namespace b200
