// The gated delta rule of the Gated DeltaNet layers (the recurrence of transformers' torch_chunk_gated_delta_rule /
// fla's chunk_gated_delta_rule, which the reference's Qwen 3.5 graph forward calls, basal/gdn_graph.py:81-87,
// :492-493), over chunks of 64 tokens, with fp32 accuracy.
//
// Per value head, with l2-normed keys k_t, scaled queries q_t, values v_t, gates g_t <= 0 and beta_t in (0, 1), the
// state S [dk = 128, dv = 128] follows S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T and the
// output is o_t = S_t^T q_t. Over a chunk with cumulative gates G (G_i = g_1 + .. + g_i within the chunk):
//   A_ij = beta_i (k_i . k_j) e^{G_i - G_j} (j < i), T = (I + A)^-1 (unit lower triangular)
//   U = T (beta V),  W = T (beta e^G K),  V' = U - W S,
//   O = e^G (Q S) + (Q K^T (.) e^{G_i - G_j}, j <= i) V',  S <- e^{G_last} S + (e^{G_last - G} K)^T V'.
//
// A CTA of 512 threads (16 warps) owns one (row, value head): its state S [128 x 128] never leaves shared memory, and
// every product of a chunk is spread over the 16 warps (16 x 16, 16 x 32 or 16 x 64 output tiles a warp). Every
// product runs on the tensor cores as mma.sync m16n8k8 with TF32 operands split in two (x = hi + lo, both TF32; each
// product is hi*hi + hi*lo + lo*hi with an fp32 accumulator, which keeps fp32 accuracy). Operands sit in shared
// memory in their natural row-major layouts, each row padded so that the fragment loads of a warp hit 32 different
// banks (leading dimensions of 4 mod 32 words for matrices read along rows, 8 mod 32 for matrices read down columns).
// Buffers are reused within a chunk: P = Q K^T takes A's place once T is found, W takes Q's once Q S and P are done
// (Q S and U stay in registers until they are used). T is found by 16 x 16 blocks: the diagonal blocks by forward
// substitution (a warp each), the off-diagonal ones by T_IJ = -T_II sum_{M = J .. I - 1} A_IM T_MJ, one block
// distance at a time.
#pragma once
#include "common.cuh"

namespace b200 {
namespace gdnchunk {

constexpr int CH = 64;     // tokens a chunk
constexpr int DK = 128;    // key dim
constexpr int DV = 128;    // value dim
constexpr int NT = 512;    // threads (16 warps)
constexpr int LK = DK + 4;  // row stride of Q, K, W (read along rows and, for K, down columns)
constexpr int LV = DV + 8;  // row stride of S and V (read down columns)
constexpr int LC = CH + 4;  // row stride of A, T, P (read along rows)
constexpr int LX = 17;      // row stride of the inverse's 16 x 16 scratch blocks

struct Params {
  const float* q;      // [rows, Hk, T, 128] (l2-normed, scaled); value head h reads key head h / (H / Hk)
  const float* k;      // [rows, Hk, T, 128] (l2-normed)
  const void* v;       // [rows, H, T, 128], fp32 or 16-bit
  const float* g;      // [rows, H, T]
  const float* beta;   // [rows, H, T]
  const float* s0;     // [s0_rows, H, 128, 128] or null (zeros); s0_rows 1 (shared) or rows
  int s0_rows;
  void* o;             // [rows, H, T, 128], fp32 or v's 16-bit type (then each value rounded once)
  float* s_out;        // [rows, H, 128, 128] or null
  int rows, Hk, H, T;
};

struct Smem {
  float S[DK * LV];      // the state [kk][c]
  float K[CH * LK];      // keys [i][kk]
  float QW[CH * LK];     // queries [i][kk]; then W = T (beta e^G K) [i][kk]
  float V[CH * LV];      // beta V, then V' = U - W S [i][c]
  float AP[CH * LC];     // A [i][j]; then P = (Q K^T (.) decay, causal) [i][j]
  float Tm[CH * LC];     // T [i][j]
  float X[4][16 * LX];   // the inverse's off-diagonal blocks X = sum A_IM T_MJ, one a warp
  float G[CH];           // cumulative gates
  float B[CH];           // beta
  float EB[CH];          // beta_i e^{G_i}
  float ED[CH];          // e^{G_last - G_i}
};

__device__ __forceinline__ void prefetch_l2(const void* a) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(a)));
}

// x rounded to TF32 (10 mantissa bits), to nearest with ties away from zero, as cvt.rna.tf32.f32 rounds a finite
// value: half a unit of the 13th bit added to the magnitude bits, the 13 bits then cleared (integer operations,
// which issue at full rate).
__device__ __forceinline__ uint32_t rna_tf32(uint32_t b) { return (b + 0x1000u) & 0xFFFFE000u; }

// x = hi + lo, both TF32 (x - hi is exact in fp32).
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = rna_tf32(__float_as_uint(x));
  lo = rna_tf32(__float_as_uint(x - __uint_as_float(hi)));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc[j] (the 16 x 8 tile at rows r0.., columns n0 + 8 j..) += sum_{k < KN} A(r, k) B(k, n) for j < NJ, one warp:
// fa(r, k) and fb(k, n) read the operands (from shared memory, scaled as the caller needs). Fragment layouts of
// m16n8k8 (g = lane / 4, t = lane % 4): A (g | g + 8, t | t + 4), B (k = t | t + 4, n = g), C (g | g + 8, 2t, 2t + 1).
template <int NJ, int KN, typename FA, typename FB>
__device__ __forceinline__ void warp_mm(float (&acc)[NJ][4], int r0, int n0, FA fa, FB fb, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll 4  // 8.51 -> 8.27 ms at C5's micro-batch; a full unroll: 12.1 ms
  for (int k0 = 0; k0 < KN; k0 += 8) {
    uint32_t ah[4], al[4];
    split_tf32(fa(r0 + g, k0 + t), ah[0], al[0]);
    split_tf32(fa(r0 + g + 8, k0 + t), ah[1], al[1]);
    split_tf32(fa(r0 + g, k0 + t + 4), ah[2], al[2]);
    split_tf32(fa(r0 + g + 8, k0 + t + 4), ah[3], al[3]);
    uint32_t bh[NJ][2], bl[NJ][2];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      split_tf32(fb(k0 + t, n0 + 8 * j + g), bh[j][0], bl[j][0]);
      split_tf32(fb(k0 + t + 4, n0 + 8 * j + g), bh[j][1], bl[j][1]);
    }
    // the three partial products as three passes over the column tiles: consecutive MMAs use different
    // accumulators (small terms first, as the sum is formed per accumulator in the same order either way)
#pragma unroll
    for (int j = 0; j < NJ; ++j) mma_tf32(acc[j], al, bh[j][0], bh[j][1]);
#pragma unroll
    for (int j = 0; j < NJ; ++j) mma_tf32(acc[j], ah, bl[j][0], bl[j][1]);
#pragma unroll
    for (int j = 0; j < NJ; ++j) mma_tf32(acc[j], ah, bh[j][0], bh[j][1]);
  }
}

template <int NJ>
__device__ __forceinline__ void zero(float (&acc)[NJ][4]) {
#pragma unroll
  for (int j = 0; j < NJ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
}

// T = (I + A)^-1 for the strictly lower A [64][64] (sh.AP) -> sh.Tm; sh.X is scratch.
__device__ __forceinline__ void unit_lower_inverse(Smem& sh, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  float* T = sh.Tm;
  const float* A = sh.AP;
  // diagonal 16 x 16 blocks: warp b, lane j < 16 owns column j of block b; rows in order
  if (warp < 4) {
    const int b0 = warp * 16;
    if (lane < 16)
      for (int i = 0; i < 16; ++i) T[(b0 + i) * LC + b0 + lane] = (i == lane) ? 1.0f : 0.0f;
    __syncwarp();
    for (int i = 1; i < 16; ++i) {
      float acc = 0.0f;
      if (lane < i) {
        for (int m = lane; m < i; ++m) acc = fmaf(A[(b0 + i) * LC + b0 + m], T[(b0 + m) * LC + b0 + lane], acc);
      }
      __syncwarp();
      if (lane < i) T[(b0 + i) * LC + b0 + lane] = -acc;
      __syncwarp();
    }
  }
  for (int e = tid; e < CH * CH; e += NT) {  // the blocks above the diagonal are zero
    const int i = e / CH, j = e % CH;
    if ((j >> 4) > (i >> 4)) T[i * LC + j] = 0.0f;
  }
  __syncthreads();
  // off-diagonal blocks, distance d = I - J: warp J a block, lane owns row lane / 2, columns (lane % 2) * 8 ..
  for (int d = 1; d < 4; ++d) {
    const int blk = warp;
    const bool on = blk + d < 4;
    const int I0 = (blk + d) * 16, J0 = blk * 16;
    const int r = lane >> 1, cb = (lane & 1) * 8;
    if (on) {
      float x[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) x[c] = 0.0f;
      for (int m = J0; m < I0; ++m) {  // X = sum_{M = J .. I - 1} A_IM T_MJ
        const float a = A[(I0 + r) * LC + m];
#pragma unroll
        for (int c = 0; c < 8; ++c) x[c] = fmaf(a, T[m * LC + J0 + cb + c], x[c]);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) sh.X[blk][r * LX + cb + c] = x[c];
    }
    __syncthreads();
    if (on) {  // T_IJ = -T_II X
      float y[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) y[c] = 0.0f;
      for (int m = 0; m < 16; ++m) {
        const float tt = T[(I0 + r) * LC + I0 + m];
#pragma unroll
        for (int c = 0; c < 8; ++c) y[c] = fmaf(tt, sh.X[blk][m * LX + cb + c], y[c]);
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) T[(I0 + r) * LC + J0 + cb + c] = -y[c];
    }
    __syncthreads();
  }
}

// Stores a warp's m16n8 accumulator tiles acc[j] (rows r0 + g, r0 + g + 8; columns n0 + 8 j + 2 t, + 1) into a
// row-major shared matrix of stride ld.
template <int NJ>
__device__ __forceinline__ void store_tiles(float* m, int ld, const float (&acc)[NJ][4], int r0, int n0, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int c = n0 + 8 * j + 2 * t;
    *reinterpret_cast<float2*>(&m[(r0 + g) * ld + c]) = make_float2(acc[j][0], acc[j][1]);
    *reinterpret_cast<float2*>(&m[(r0 + g + 8) * ld + c]) = make_float2(acc[j][2], acc[j][3]);
  }
}

// 4 consecutive values of v -> fp32
__device__ __forceinline__ float4 load_v4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
template <typename TV>
__device__ __forceinline__ float4 load_v4(const TV* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const TV* h = reinterpret_cast<const TV*>(&u);
  return make_float4(static_cast<float>(h[0]), static_cast<float>(h[1]), static_cast<float>(h[2]),
                     static_cast<float>(h[3]));
}

__device__ __forceinline__ void store2(float* d, float a, float b) {
  *reinterpret_cast<float2*>(d) = make_float2(a, b);
}
template <typename TO>
__device__ __forceinline__ void store2(TO* d, float a, float b) {
  TO h[2] = {static_cast<TO>(a), static_cast<TO>(b)};
  *reinterpret_cast<uint32_t*>(d) = *reinterpret_cast<const uint32_t*>(h);
}

template <typename TV, typename TO>
__global__ void __launch_bounds__(NT, 1) gdn_chunk_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sh = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int rh = blockIdx.x;  // r * H + h
  const int r = rh / p.H, h = rh % p.H;
  const int64_t base = (int64_t)rh * p.T;  // token row of (r, h, t = 0) in v / o, and in g / beta
  const int64_t base_qk = ((int64_t)r * p.Hk + h / (p.H / p.Hk)) * p.T;  // ... in q / k (its key head)
  const TV* vsrc = static_cast<const TV*>(p.v);
  pdl_wait();
  for (int e = tid * 4; e < DK * DV; e += NT * 4) {  // the initial state
    const int kk = e / DV, c = e % DV;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.s0) {
      const int sr = p.s0_rows == 1 ? 0 : r;
      s = *reinterpret_cast<const float4*>(p.s0 + (((int64_t)sr * p.H + h) * DK + kk) * DV + c);
    }
    *reinterpret_cast<float4*>(&sh.S[kk * LV + c]) = s;
  }
  // this warp's tiles: 64 x 64 products 16 rows x 16 columns (NJ = 2), 64 x 128 products 16 x 32 (NJ = 4), the
  // 128 x 128 state update 16 x 64 (NJ = 8)
  const int rt = (warp >> 2) * 16, n16 = (warp & 3) * 16, n32 = (warp & 3) * 32;
  const int rs = (warp >> 1) * 16, n64 = (warp & 1) * 64;
  for (int t0 = 0; t0 < p.T; t0 += CH) {
    const int n = min(CH, p.T - t0);
    // ---- chunk loads: K and Q row-major, beta, G ----
    for (int e = tid; e < CH * DK / 4; e += NT) {
      const int i = e / (DK / 4), f = e % (DK / 4);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), qv = kv;
      if (i < n) {
        kv = __ldg(reinterpret_cast<const float4*>(p.k + (base_qk + t0 + i) * DK) + f);
        qv = __ldg(reinterpret_cast<const float4*>(p.q + (base_qk + t0 + i) * DK) + f);
      }
      *reinterpret_cast<float4*>(&sh.K[i * LK + 4 * f]) = kv;
      *reinterpret_cast<float4*>(&sh.QW[i * LK + 4 * f]) = qv;
    }
    if (tid < CH) {
      sh.B[tid] = tid < n ? __ldg(p.beta + base + t0 + tid) : 0.0f;
      sh.G[tid] = tid < n ? __ldg(p.g + base + t0 + tid) : 0.0f;
    }
    {  // ask L2 for the next chunk's keys, queries and values (128-byte lines), so its loads do not wait for DRAM
      const int n2 = min(CH, p.T - t0 - CH);
      constexpr int VL = DV * (int)sizeof(TV) / 128;  // lines of a value row
      for (int e = tid; e < n2 * (8 + VL); e += NT) {
        const int i = e / (8 + VL), l = e % (8 + VL);
        if (l < 8) {
          prefetch_l2((l < 4 ? p.k : p.q) + (base_qk + t0 + CH + i) * DK + (l % 4) * 32);
        } else {
          prefetch_l2(vsrc + (base + t0 + CH + i) * DV + (l - 8) * (128 / (int)sizeof(TV)));
        }
      }
    }
    __syncthreads();
    if (tid == 0) {  // cumulative gates, in token order
      float acc = 0.0f;
      for (int i = 0; i < CH; ++i) {
        acc += sh.G[i];
        sh.G[i] = acc;
      }
    }
    for (int e = tid; e < CH * DV / 4; e += NT) {  // beta V
      const int i = e / (DV / 4), f = e % (DV / 4);
      float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n) {
        val = load_v4(vsrc + (base + t0 + i) * DV + 4 * f);
        const float bt = sh.B[i];
        val.x *= bt;
        val.y *= bt;
        val.z *= bt;
        val.w *= bt;
      }
      *reinterpret_cast<float4*>(&sh.V[i * LV + 4 * f]) = val;
    }
    __syncthreads();
    if (tid < CH) {  // read after the inverse's barriers
      sh.EB[tid] = sh.B[tid] * expf(sh.G[tid]);
      sh.ED[tid] = expf(sh.G[CH - 1] - sh.G[tid]);
    }
    // ---- A_ij = beta_i (k_i . k_j) e^{G_i - G_j} for j < i ----
    {
      float kk[2][4];
      zero(kk);
      warp_mm<2, DK>(kk, rt, n16, [&](int i, int c) { return sh.K[i * LK + c]; },
                     [&](int c, int j) { return sh.K[j * LK + c]; }, lane);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = rt + g8 + (e >> 1) * 8, jj = n16 + 8 * j + 2 * t4 + (e & 1);
          sh.AP[i * LC + jj] = jj < i ? sh.B[i] * kk[j][e] * expf(sh.G[i] - sh.G[jj]) : 0.0f;
        }
    }
    __syncthreads();
    unit_lower_inverse(sh, tid);  // ends with a barrier; A is not read again
    // ---- P = (q_i . k_j) e^{G_i - G_j} for j <= i (into A's place) ----
    {
      float qk[2][4];
      zero(qk);
      warp_mm<2, DK>(qk, rt, n16, [&](int i, int c) { return sh.QW[i * LK + c]; },
                     [&](int c, int j) { return sh.K[j * LK + c]; }, lane);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = rt + g8 + (e >> 1) * 8, jj = n16 + 8 * j + 2 * t4 + (e & 1);
          sh.AP[i * LC + jj] = jj <= i ? qk[j][e] * expf(sh.G[i] - sh.G[jj]) : 0.0f;
        }
    }
    // ---- Q S and U = T (beta V) [64 x 128], kept in registers ----
    float qs[4][4], u[4][4];
    zero(qs);
    zero(u);
    warp_mm<4, DK>(qs, rt, n32, [&](int i, int k) { return sh.QW[i * LK + k]; },
                   [&](int k, int c) { return sh.S[k * LV + c]; }, lane);
    warp_mm<4, CH>(u, rt, n32, [&](int i, int k) { return sh.Tm[i * LC + k]; },
                   [&](int k, int c) { return sh.V[k * LV + c]; }, lane);
    __syncthreads();  // every read of Q is done (P, Q S)
    // ---- W = T (beta e^G K) [64 x 128] (into Q's place) ----
    {
      float w[4][4];
      zero(w);
      warp_mm<4, CH>(w, rt, n32, [&](int i, int k) { return sh.Tm[i * LC + k]; },
                     [&](int k, int c) { return sh.K[k * LK + c] * sh.EB[k]; }, lane);
      store_tiles(sh.QW, LK, w, rt, n32, lane);
    }
    __syncthreads();  // W and P are complete; every read of beta V is done (U)
    // ---- V' = U - W S [64 x 128] (into V) ----
    {
      float ws[4][4];
      zero(ws);
      warp_mm<4, DK>(ws, rt, n32, [&](int i, int k) { return sh.QW[i * LK + k]; },
                     [&](int k, int c) { return sh.S[k * LV + c]; }, lane);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) u[j][e] -= ws[j][e];
      store_tiles(sh.V, LV, u, rt, n32, lane);
    }
    __syncthreads();
    // ---- O = e^G (Q S) + P V' ----
    {
      float pv[4][4];
      zero(pv);
      warp_mm<4, CH>(pv, rt, n32, [&](int i, int k) { return sh.AP[i * LC + k]; },
                     [&](int k, int c) { return sh.V[k * LV + c]; }, lane);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = rt + g8 + hh * 8;
        if (i < n) {
          const float eg = expf(sh.G[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = n32 + 8 * j + 2 * t4;
            store2(static_cast<TO*>(p.o) + (base + t0 + i) * DV + c, fmaf(eg, qs[j][2 * hh], pv[j][2 * hh]),
                   fmaf(eg, qs[j][2 * hh + 1], pv[j][2 * hh + 1]));
          }
        }
      }
    }
    // ---- S <- e^{G_last} S + (e^{G_last - G} K)^T V' [128 x 128] ----
    {
      const float gl = sh.G[CH - 1];
      float sn[8][4];
      zero(sn);
      warp_mm<8, CH>(sn, rs, n64, [&](int kk, int i) { return sh.K[i * LK + kk] * sh.ED[i]; },
                     [&](int i, int c) { return sh.V[i * LV + c]; }, lane);
      const float egl = expf(gl);
      float old[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) old[j][e] = sh.S[(rs + g8 + (e >> 1) * 8) * LV + n64 + 8 * j + 2 * t4 + (e & 1)];
      __syncthreads();  // every thread has read S (W S, Q S) and its own entries of it
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sh.S[(rs + g8 + (e >> 1) * 8) * LV + n64 + 8 * j + 2 * t4 + (e & 1)] = fmaf(egl, old[j][e], sn[j][e]);
    }
    __syncthreads();
  }
  if (p.s_out) {
    for (int e = tid * 4; e < DK * DV; e += NT * 4) {
      const int kk = e / DV, c = e % DV;
      *reinterpret_cast<float4*>(p.s_out + ((int64_t)rh * DK + kk) * DV + c) =
          *reinterpret_cast<const float4*>(&sh.S[kk * LV + c]);
    }
  }
  pdl_launch();
}

}  // namespace gdnchunk
}  // namespace b200
