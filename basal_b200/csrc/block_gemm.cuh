// The block-scaled GEMM of the FP8-block and INT8-block formats on sm_100a (replaces the Triton kernel of
// basal/blockquant.py:63-106):
//
//   C[m, n] = sum_kb (A_kb[m, :] . B_kb[n, :]) * a_s[m, kb] * b_s[n / 128, kb]        (kb: 128-deep slices of K)
//
// A [M, K] and B [N, K] are 8-bit, K-major. One persistent CTA per SM walks 128 x 256 output tiles (static round
// robin, the 256-wide weight tiles of one 128-row activation tile next to each other). Its warps:
//   warp 0      TMA producer: A and B slices of 128 bytes of K into a shared-memory ring (128-byte swizzle), 3
//               stages for 16-bit outputs, 4 for fp32
//   warp 1      MMA issuer: 4 x tcgen05.mma (K = 32 each) per slice into one of two TMEM accumulators of 256
//               columns (kind::f8f6f4 e4m3 -> f32, or kind::i8 s8 -> s32, exact for a 128-deep slice)
//   warp 2      TMEM allocation (512 columns) and release
//   warps 4-11  promotion: per slice, tcgen05.ld of the slice's product (64 columns in flight per wait), times
//               a_s * b_s, added into fp32 registers with packed f32x2 FMAs (128 columns a thread); after the last
//               slice, the cast (and bias); 16-bit outputs go through a 64 KB staging buffer (128-byte swizzle) and
//               asynchronous TMA stores (rows past M clipped by the tensor map), so the promotion of the next tile
//               starts at once; fp32 outputs are stored directly
// The MMA of slice kb + 1 runs while the promotion reads slice kb from the other accumulator. The producer warpgroup
// gives registers to the promotion warpgroups (setmaxnreg: 40 / 232 of the 168 a thread at launch). A row's result
// never depends on the other rows (no split of K, the same slice order for every M).
#pragma once
#include "quant.cuh"

namespace b200 {
namespace blockgemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes (= elements) of K per stage: one scale slice
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr uint32_t STAGE_TX = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr int NUM_EPI_WARPS = 8;
constexpr uint32_t TMEM_COLS = 512;
// setmaxnreg split: 128 producer-warpgroup threads at REGS_LOW, 256 promotion threads at REGS_HIGH; the launch must
// hold LAUNCH_REGS a thread (checked on the host before every first launch: a split beyond the launch's registers
// would wait forever)
constexpr uint32_t REGS_LOW = 40, REGS_HIGH = 232;
constexpr uint32_t LAUNCH_REGS = (REGS_LOW * 128 + REGS_HIGH * 256) / NUM_THREADS;
static_assert(REGS_LOW * 128 + REGS_HIGH * 256 <= LAUNCH_REGS * NUM_THREADS, "register split");

constexpr int SUB_BYTES = BM * 128;  // one 64-column x 128-row sub-tile of 16-bit outputs (128-byte swizzle)

// Shared memory of one CTA: the stage ring, the output staging (16-bit outputs), the barriers.
template <int STAGES_, bool STAGING_>
struct Smem {
  static constexpr int STAGES = STAGES_;
  static constexpr bool STAGING = STAGING_;
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint8_t out[STAGING ? 4 : 1][STAGING ? SUB_BYTES : 1024];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t rfull[2];  // residual epilogue: each warpgroup's residual tile has landed in its staging sub-tiles
  uint64_t mdrain;
  uint32_t tmem_base;
  int abort;
};
template <int OUT>
using SmemOf = Smem<OUT == BASAL200_F32 ? 4 : 3, OUT != BASAL200_F32>;
template <int OUT>
constexpr size_t smem_bytes() {
  return sizeof(SmemOf<OUT>) + 1024;
}

struct Params {
  const float* s;   // [M, K/128]
  const float* ws;  // [N/128, K/128]
  const void* bias; // [N] in the output type, or null
  void* c;          // [M, N] (fp32 outputs, stored directly)
  int M, N, nkb, tiles_n, num_tiles;
  int npeers;       // 16-bit outputs: the output buffers the tiles are stored into (OutMaps), 1 or, for a column-
  int col_off;      // parallel linear gathered on the fly, every rank's [M, n_total] output, at column col_off
  int glu_up;       // gated linear (ACT != 0): the weight rows [gate; up] with up from row glu_up (= the output width)
  const uint32_t* gate = nullptr;  // gathered linear: this rank's peer-barrier status word (or null); non-zero = store nothing
};

// The number of output buffers a GEMM stores into: none when the peer barrier before a gathered GEMM recorded a
// timeout (a rank that missed the barrier must not write into a peer's output while the peer may still read it).
// Read after pdl_wait: the barrier kernel has completed and its store is visible.
__device__ __forceinline__ int stored_peers(int npeers, const uint32_t* gate) {
  if (gate && *reinterpret_cast<const volatile uint32_t*>(gate) != 0u) return 0;
  return npeers;
}

// Gated-linear activations of the fused gate/up epilogue, in fp32 on the 16-bit-rounded gate, with the formulas and
// operation order of torch's CUDA kernels (so that the cast result matches the unfused ops'): silu(x) = x / (1 +
// e^-x); gelu, tanh form: 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))).
enum { kActNone = 0, kActSilu = 1, kActGeluTanh = 2 };
template <int ACT>
__device__ __forceinline__ float glu_act(float x) {
  if (ACT == kActSilu) return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
  const float cube = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, cube)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// The tensor maps of the output buffers of a 16-bit output: one for a plain GEMM; one per rank for a GEMM whose
// column shard is stored straight into every rank's full output (the all-gather of a column-parallel linear done by
// the epilogue's TMA stores over NVLink, one plain store per rank and sub-tile).
constexpr int kMaxPeers = 8;
struct OutMaps {
  CUtensorMap m[kMaxPeers];
};

// ---------------------------------------------------------------------------------------------------------------
// Peer barrier over peer-mapped signal pads: word r of rank q's pad holds the last call number rank r reached, word
// kMaxPeers this rank's own call count, word kPadStatus a sticky status (0 = every barrier so far completed).
// Thread r stores the call number into rank r's pad (release, system scope) and waits for rank r's (acquire), giving
// up after timeout_ns with a fault bit. A rank whose status is set (a wait of this or an earlier call gave up, or a
// peer's did) writes it into every peer's status word too, so every rank's gathered GEMMs stop storing and every
// rank's host sees the failure.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kPadStatus = kMaxPeers + 1;
struct PeerPads {
  uint32_t* p[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerPads pads, int world, int rank,
                                                          long long timeout_ns) {
  __shared__ uint32_t call;
  if (threadIdx.x == 0) {
    call = pads.p[rank][kMaxPeers] + 1;  // only this rank's stream touches its count
    pads.p[rank][kMaxPeers] = call;
  }
  __syncthreads();
  const int r = threadIdx.x;
  __shared__ int timed_out;
  if (r == 0) timed_out = 0;
  __syncthreads();
  if (r < world) {
    __threadfence_system();
    st_release_sys(pads.p[r] + rank, call);
    const unsigned long long t0 = globaltimer();
    while ((int)(ld_acquire_sys(pads.p[rank] + r) - call) < 0) {
      if (globaltimer() - t0 > (unsigned long long)timeout_ns) {
        atomicOr(&g_fault, kFaultTimeoutPeer);
        timed_out = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (timed_out && r == 0) pads.p[rank][kPadStatus] = 1u;
  __syncthreads();
  const uint32_t status = *reinterpret_cast<volatile uint32_t*>(pads.p[rank] + kPadStatus);
  if (status != 0u && r < world && r != rank) st_release_sys(pads.p[r] + kPadStatus, status);
}

// Bounded drain wait (the abort flag is already set when it runs).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(&g_fault, kFaultTimeoutDrain);
      return;
    }
  }
}

// Offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled sub-tile (the layout TMA reads with
// CU_TENSOR_MAP_SWIZZLE_128B).
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// All 32 lanes wait; the warp proceeds only if every lane saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned fault) {
  const bool ok = mbar_wait(bar, parity, abort_flag, fault);
  return __all_sync(0xffffffffu, ok);
}

// Casts and stores of fp32 results: pack casts the PER values of one 16-byte chunk, vec8 writes 8 consecutive
// outputs (one 16- or 32-byte store); a bias in the output type is added to the cast value and rounded again, as
// torch adds a bias to the cast product.
template <int OUT>
struct Store;
template <>
struct Store<BASAL200_BF16> {
  using T = __nv_bfloat16;
  static constexpr int PER = 8;
  __device__ __forceinline__ static uint4 pack(const float* v, const T* bias) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      if (bias) {
        const float2 y = __bfloat1622float2(h);
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + 2 * i));
        h = __floats2bfloat162_rn(__fadd_rn(y.x, b.x), __fadd_rn(y.y, b.y));
      }
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return u;
  }
  __device__ __forceinline__ static void vec8(T* dst, const float* v, const T* bias) {
    *reinterpret_cast<uint4*>(dst) = pack(v, bias);
  }
};
template <>
struct Store<BASAL200_F16> {
  using T = __half;
  static constexpr int PER = 8;
  __device__ __forceinline__ static uint4 pack(const float* v, const T* bias) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      if (bias) {
        const float2 y = __half22float2(h);
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(bias + 2 * i));
        h = __floats2half2_rn(__fadd_rn(y.x, b.x), __fadd_rn(y.y, b.y));
      }
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return u;
  }
  __device__ __forceinline__ static void vec8(T* dst, const float* v, const T* bias) {
    *reinterpret_cast<uint4*>(dst) = pack(v, bias);
  }
};
template <>
struct Store<BASAL200_F32> {
  using T = float;
  static constexpr int PER = 4;
  __device__ __forceinline__ static uint4 pack(const float* v, const T* bias) {
    float4 f = make_float4(v[0], v[1], v[2], v[3]);
    if (bias) {
      f.x = __fadd_rn(f.x, bias[0]);
      f.y = __fadd_rn(f.y, bias[1]);
      f.z = __fadd_rn(f.z, bias[2]);
      f.w = __fadd_rn(f.w, bias[3]);
    }
    return make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
  }
  __device__ __forceinline__ static void vec8(T* dst, const float* v, const T* bias) {
    *reinterpret_cast<uint4*>(dst) = pack(v, bias);
    *reinterpret_cast<uint4*>(dst + 4) = pack(v + 4, bias ? bias + 4 : nullptr);
  }
};

// The gated linear's second step for few rows: y [M, I] = act(gate) * up from the merged linear's 16-bit output
// t [M, 2I] (gate columns 0 .. I-1, up I .. 2I-1), 8 outputs a thread, the same arithmetic as glu_apply.
template <int OUT, int ACT>
__global__ void __launch_bounds__(256) glu_rows_kernel(const void* __restrict__ t, void* __restrict__ y, int64_t M,
                                                       int64_t I) {
  using OutT = typename Store<OUT>::T;
  pdl_launch();
  pdl_wait();
  const int64_t idx = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 8;  // first output of this thread
  if (idx >= M * I) return;
  const int64_t m = idx / I, c = idx - m * I;
  const OutT* tr = static_cast<const OutT*>(t) + m * 2 * I;
  const uint4 gw = *reinterpret_cast<const uint4*>(tr + c);
  const uint4 uw = *reinterpret_cast<const uint4*>(tr + I + c);
  const OutT* gh = reinterpret_cast<const OutT*>(&gw);
  const OutT* uh = reinterpret_cast<const OutT*>(&uw);
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = static_cast<float>(static_cast<OutT>(glu_act<ACT>(static_cast<float>(gh[e]))));
    v[e] = __fmul_rn(a, static_cast<float>(uh[e]));
  }
  Store<OUT>::vec8(static_cast<OutT*>(y) + idx, v, nullptr);
}

// The residual linear's second step for few rows: y = t + residual (both 16-bit, [n] elements, 8 a thread), rounded
// as torch adds two 16-bit tensors; y may be the residual itself.
template <int OUT>
__global__ void __launch_bounds__(256) add_rows_kernel(const void* __restrict__ t, const void* res, void* y,
                                                       int64_t n) {
  using OutT = typename Store<OUT>::T;
  pdl_launch();
  pdl_wait();
  const int64_t idx = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 8;
  if (idx >= n) return;
  const uint4 tw = *reinterpret_cast<const uint4*>(static_cast<const OutT*>(t) + idx);
  const uint4 rw = *reinterpret_cast<const uint4*>(static_cast<const OutT*>(res) + idx);
  const OutT* th = reinterpret_cast<const OutT*>(&tw);
  const OutT* rh = reinterpret_cast<const OutT*>(&rw);
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(static_cast<float>(th[e]), static_cast<float>(rh[e]));
  Store<OUT>::vec8(static_cast<OutT*>(y) + idx, v, nullptr);
}

// The gated epilogue's two steps for one promotion thread (row r of the tile, 128 accumulator columns as packed
// pairs): glu_send casts the 64 columns from group J0 (8 columns a group) into a staging sub-tile for the other
// warpgroup; glu_apply combines this thread's 64 columns from group J0 with the other warpgroup's cast values
// (`other`) into act(gate) * up, stored into sub-tile `dst` (OWN_GATE: this thread holds the gate).
template <int OUT, int J0>
__device__ __forceinline__ void glu_send(const uint64_t (&acc)[64], uint8_t* sub, int r) {
  using OutT = typename Store<OUT>::T;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_f2(acc[(J0 + j) * 4 + i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    Store<OUT>::vec8(reinterpret_cast<OutT*>(sub + sw128(r, j)), v, nullptr);
  }
}

template <int OUT, int ACT, int J0, bool OWN_GATE>
__device__ __forceinline__ void glu_apply(const uint64_t (&acc)[64], const uint8_t* other, uint8_t* dst, int r) {
  using OutT = typename Store<OUT>::T;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float own[8], y[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_f2(acc[(J0 + j) * 4 + i]);
      own[2 * i] = f.x;
      own[2 * i + 1] = f.y;
    }
    const uint4 ow = Store<OUT>::pack(own, nullptr);  // this thread's linear output, cast
    const uint4 xw = *reinterpret_cast<const uint4*>(other + sw128(r, j));
    const OutT* gh = reinterpret_cast<const OutT*>(OWN_GATE ? &ow : &xw);
    const OutT* uh = reinterpret_cast<const OutT*>(OWN_GATE ? &xw : &ow);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = static_cast<float>(static_cast<OutT>(glu_act<ACT>(static_cast<float>(gh[e]))));
      y[e] = __fmul_rn(a, static_cast<float>(uh[e]));
    }
    Store<OUT>::vec8(reinterpret_cast<OutT*>(dst + sw128(r, j)), y, nullptr);
  }
}

// Redistributes a warp's 32 rows x CH chunks of 16 bytes (CH = 8 or 4; lane = row, c[j] = chunk j) so that lane L
// holds in c[i] chunk L % CH of row (32 / CH) i + L / CH, and a store of c[i] by the warp writes 32 / CH whole row
// segments of 16 CH bytes: log2(CH) shuffle exchanges of a chunk-index bit with a lane bit (chunk bit k with lane
// bit 5 - log2(CH) + k), then one fixed lane rotation.
template <int CH>
__device__ __forceinline__ void rows_to_segments(uint4 (&c)[CH], int lane) {
  static_assert(CH == 4 || CH == 8, "4 or 8 chunks a row");
  constexpr int LCH = CH == 8 ? 3 : 2;
#pragma unroll
  for (int k = 0; k < LCH; ++k) {
    const int m = 1 << (5 - LCH + k);
    const bool hi = lane & m;
#pragma unroll
    for (int s = 0; s < CH; ++s) {
      if (s & (1 << k)) continue;
      const int t = s | (1 << k);
      const uint4 send = hi ? c[s] : c[t];
      uint4 recv;
      recv.x = __shfl_xor_sync(0xffffffffu, send.x, m);
      recv.y = __shfl_xor_sync(0xffffffffu, send.y, m);
      recv.z = __shfl_xor_sync(0xffffffffu, send.z, m);
      recv.w = __shfl_xor_sync(0xffffffffu, send.w, m);
      if (hi)
        c[s] = recv;
      else
        c[t] = recv;
    }
  }
  const int src = ((lane & (CH - 1)) << (5 - LCH)) | (lane >> LCH);
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    c[s].x = __shfl_sync(0xffffffffu, c[s].x, src);
    c[s].y = __shfl_sync(0xffffffffu, c[s].y, src);
    c[s].z = __shfl_sync(0xffffffffu, c[s].z, src);
    c[s].w = __shfl_sync(0xffffffffu, c[s].w, src);
  }
}

// ACT != kActNone: the gated linear y = act(x W_gate^T) * (x W_up^T) of a merged [gate; up] weight (up from row
// p.glu_up), for 16-bit outputs: a 256-wide tile holds gate block tn (accumulator columns 0-127, loaded as one
// 128-row box) and up block tn (columns 128-255). The two promotion warpgroups trade half of their cast values
// through the staging buffer, each computes act(gate) * up for 64 columns with the roundings of the unfused torch ops
// (each linear output cast, act(.) cast, the product cast), and one 128-column output tile is stored.
// RES: y = residual + (the linear's output cast, + bias), rounded as torch adds two 16-bit tensors; the residual
// [M, N] is read through out.m[1] (the output's box), its tile TMA-loaded into the staging sub-tiles in the middle of
// the tile's slices, added in place and stored (so y may be the residual itself).
template <bool INT8, int OUT, int ACT = kActNone, bool RES = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    block_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ OutMaps out, const Params p) {
  static_assert(ACT == kActNone || OUT != BASAL200_F32, "the gated linear stores 16-bit outputs");
  static_assert(!RES || (ACT == kActNone && OUT != BASAL200_F32), "the residual epilogue: 16-bit plain linears");
  using S = SmemOf<OUT>;
  constexpr int STAGES = S::STAGES;
  extern __shared__ uint8_t smem_raw[];
  S& sh = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.tfull[b], 1);
      mbar_init(&sh.tempty[b], NUM_EPI_WARPS);
      mbar_init(&sh.rfull[b], 1);
    }
    mbar_init(&sh.mdrain, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (S::STAGING)
      for (int r = 0; r < p.npeers; ++r) tma_prefetch_desc(&out.m[r]);
    if (RES) tma_prefetch_desc(&out.m[1]);
  }
  if (warp == 2) tmem_alloc(&sh.tmem_base, TMEM_COLS);
  pdl_launch();
  pdl_wait();  // the set-up above ran while the kernel before this one finished
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  if (warp < EPI_WARP0) regs_release<REGS_LOW>();
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0, last_phase = 0;  // per-stage bit masks, for the drain after an abort
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
        for (int kb = 0; kb < p.nkb; ++kb) {
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, abort_flag, kFaultTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.full[stage], STAGE_TX);
          tma_load_2d(sh.a[stage], &tmA, &sh.full[stage], kb * BK, tm * BM);
          if (ACT != kActNone) {  // gate block tn, then up block tn (tmB's box: 128 rows)
            tma_load_2d(sh.b[stage], &tmB, &sh.full[stage], kb * BK, tn * 128);
            tma_load_2d(sh.b[stage] + B_BYTES / 2, &tmB, &sh.full[stage], kb * BK, p.glu_up + tn * 128);
          } else {
            tma_load_2d(sh.b[stage], &tmB, &sh.full[stage], kb * BK, tn * BN);
          }
          filled |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let the copies already issued land before the CTA's shared memory goes away
        for (int s = 0; s < STAGES; ++s)
          if (filled & (1u << s)) drain_wait(&sh.full[s], (last_phase >> s) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = INT8 ? idesc_dense(2, 1, 1, BM, BN) : idesc_dense(1, 0, 0, BM, BN);
      int stage = 0;
      uint32_t phase = 0, acc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int kb = 0; kb < p.nkb; ++kb) {
          const uint32_t buf = acc & 1, aph = (acc >> 1) & 1;
          if (!mbar_wait(&sh.tempty[buf], aph ^ 1, abort_flag, kFaultTimeoutMma) ||
              !mbar_wait(&sh.full[stage], phase, abort_flag, kFaultTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + buf * BN;
          const uint64_t ad = desc_sw128(smem_u32(sh.a[stage]));
          const uint64_t bd = desc_sw128(smem_u32(sh.b[stage]));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            if (INT8)
              mma_i8(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
            else
              mma_f8f6f4(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
          }
          mma_commit(&sh.empty[stage]);
          mma_commit(&sh.tfull[buf]);
          ++acc;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // every MMA issued has finished before TMEM and shared memory are released
      mma_commit(&sh.mdrain);
      drain_wait(&sh.mdrain, 0);
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- promotion and epilogue ----------------
    regs_claim<REGS_HIGH>();
    using OutT = typename Store<OUT>::T;
    const int ew = warp - EPI_WARP0;
    const int half = ew >> 2;        // which 128 columns of the 256-wide tile
    const int quad = warp & 3;       // the TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;  // row within the tile
    const bool issuer = (ew & 3) == 0 && lane == 0;
    const int nkb = p.nkb;
    const int npeers = stored_peers(p.npeers, p.gate);  // after pdl_wait (above)
    uint32_t acc_cnt = 0;
    bool ok = true;
    uint32_t res_phase = 0;    // residual epilogue: tiles of this warpgroup so far (the rfull phase)
    bool res_pending = false;  // the issuer's residual load not yet waited for
    const int res_kb = nkb / 2;  // the slice at whose start the residual tile is requested (mid-tile: time to land)
    // this thread's activation-scale row and weight-scale block of a tile
    auto scale_rows = [&](int t, const float*& srow, const float*& wsr) {
      const int tm = t / p.tiles_n, tn = t - tm * p.tiles_n;
      const int n0 = ACT != kActNone ? tn * 128 : tn * BN + half * 128;
      srow = p.s + (int64_t)min(tm * BM + r, p.M - 1) * nkb;
      const int wblk = ACT != kActNone ? (half ? p.glu_up / 128 + tn : tn) : min(n0 / 128, p.N / 128 - 1);
      wsr = p.ws + (int64_t)wblk * nkb;
    };
    // the first slice's scales of the next tile are loaded during the last slice of this one (not at its start,
    // where their round trip would hold up the promotion of slice 0)
    float sa_next = 0.0f, sb_next = 0.0f;
    if ((int)blockIdx.x < p.num_tiles) {
      const float *sr0, *ws0;
      scale_rows(blockIdx.x, sr0, ws0);
      sa_next = __ldg(sr0);
      sb_next = __ldg(ws0);
    }
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      const int row = tm * BM + r;
      const int n0 = ACT != kActNone ? tn * 128 : tn * BN + half * 128;  // gated: the output columns of the tile
      const bool nvalid = n0 < p.N;
      const float *srow, *wsr;
      scale_rows(tile, srow, wsr);
      uint64_t acc[64];  // 128 fp32 accumulators as packed pairs
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0ull;
      float sa = sa_next, sb = sb_next;
      for (int kb = 0; ok && kb < nkb; ++kb) {
        const float sc = sa * sb;
        const uint64_t sc2 = pack_f2(sc, sc);
        if (kb + 1 < nkb) {
          sa = __ldg(srow + kb + 1);
          sb = __ldg(wsr + kb + 1);
        } else if (tile + (int)gridDim.x < p.num_tiles) {
          const float *srn, *wsn;
          scale_rows(tile + gridDim.x, srn, wsn);
          sa_next = __ldg(srn);
          sb_next = __ldg(wsn);
        }
        if (RES && kb == res_kb && issuer) {  // the residual tile into this half's staging sub-tiles
          tma_store_wait_read();  // the previous tile's stores have read them
          if (nvalid) {
            mbar_arrive_expect_tx(&sh.rfull[half], 2 * SUB_BYTES);
            tma_load_2d(sh.out[half * 2], &out.m[1], &sh.rfull[half], n0, tm * BM);
            tma_load_2d(sh.out[half * 2 + 1], &out.m[1], &sh.rfull[half], n0 + 64, tm * BM);
          } else {
            mbar_arrive(&sh.rfull[half]);
          }
          res_pending = true;
        }
        const uint32_t buf = acc_cnt & 1, ph = (acc_cnt >> 1) & 1;
        if (!warp_wait(&sh.tfull[buf], ph, abort_flag, kFaultTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * BN + half * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 64 columns in flight per wait
          uint64_t x[32];
          tmem_ld64_pairs<INT8>(taddr + h * 64, x);
          if (h == 1) {  // every read of this accumulator is done: hand it back to the MMA before the FMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.tempty[buf]);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) ffma2p(acc[h * 32 + j], x[j], sc2);
        }
        ++acc_cnt;
      }
      const OutT* bias = (p.bias && nvalid) ? reinterpret_cast<const OutT*>(p.bias) + n0 : nullptr;
      if constexpr (ACT != kActNone) {
        // the up half casts its values into its two staging sub-tiles; the gate half turns them into the output.
        // Both halves take every barrier below, so they agree on going on first (all 256 promotion threads).
        if (issuer) tma_store_wait_read();     // the previous tile's stores have read the staging
        ok = named_barrier_and(3, 256, ok);
        if (!ok) break;
        // each half activates 64 of the tile's 128 output columns: the gate half columns 0-63 (sub-tile 0), the up
        // half 64-127 (sub-tile 1); first each casts the values the other half needs into staging sub-tile 2 (up,
        // columns 0-63) or 3 (gate, columns 64-127). (Constant register indices in both branches: an index that
        // depends on the half would put the accumulators in local memory.)
        if (half) {
          glu_send<OUT, 0>(acc, sh.out[2], r);
        } else {
          glu_send<OUT, 8>(acc, sh.out[3], r);
        }
        named_barrier(4, 256);  // the exchanged values are in shared memory
        if (half) {
          glu_apply<OUT, ACT, 8, false>(acc, sh.out[3], sh.out[1], r);
        } else {
          glu_apply<OUT, ACT, 0, true>(acc, sh.out[2], sh.out[0], r);
        }
        fence_proxy_async();
        named_barrier(5, 256);  // both halves have read the exchanged values and written the output tile
        if (half == 0 && issuer) {
          for (int q = 0; q < npeers; ++q) {
            tma_store_2d(&out.m[q], sh.out[0], p.col_off + n0, tm * BM);
            tma_store_2d(&out.m[q], sh.out[1], p.col_off + n0 + 64, tm * BM);
          }
          tma_store_commit();
        }
      } else if constexpr (S::STAGING) {
        // cast (+ bias) into this half's two staging sub-tiles, then two TMA stores of 128 rows x 64 columns
        if (issuer) tma_store_wait_read();          // the previous tile's stores have read the staging
        if (RES && ok) ok = mbar_wait(&sh.rfull[half], res_phase & 1, abort_flag, kFaultTimeoutEpilogue);
        ok = named_barrier_and(1 + half, 128, ok);  // the warpgroup agrees whether to go on
        if (!ok) break;
        if (RES) {
          ++res_phase;
          res_pending = false;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack_f2(acc[j * 4 + i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
          }
          OutT* dst = reinterpret_cast<OutT*>(sh.out[half * 2 + (j >> 3)] + sw128(r, j & 7));
          if (RES) {  // the linear's output as torch casts it (+ bias), then + the residual, cast again
            const uint4 lw = Store<OUT>::pack(v, bias ? bias + j * 8 : nullptr);
            const uint4 rw = *reinterpret_cast<const uint4*>(dst);
            const OutT* lh = reinterpret_cast<const OutT*>(&lw);
            const OutT* rh = reinterpret_cast<const OutT*>(&rw);
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(static_cast<float>(lh[e]), static_cast<float>(rh[e]));
            Store<OUT>::vec8(dst, y, nullptr);
          } else {
            Store<OUT>::vec8(dst, v, bias ? bias + j * 8 : nullptr);
          }
        }
        fence_proxy_async();
        named_barrier(1 + half, 128);
        if (issuer) {
          if (nvalid) {
            for (int r = 0; r < npeers; ++r) {
              tma_store_2d(&out.m[r], sh.out[half * 2], p.col_off + n0, tm * BM);
              tma_store_2d(&out.m[r], sh.out[half * 2 + 1], p.col_off + n0 + 64, tm * BM);
            }
          }
          tma_store_commit();
        }
      } else {
        if (!ok) break;
        if (nvalid && row < p.M) {
          OutT* dst = reinterpret_cast<OutT*>(p.c) + (int64_t)row * p.N + n0;
#pragma unroll
          for (int c = 0; c < 128; c += 8) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = unpack_f2(acc[c / 2 + i]);
              v[2 * i] = f.x;
              v[2 * i + 1] = f.y;
            }
            Store<OUT>::vec8(dst + c, v, bias ? bias + c : nullptr);
          }
        }
      }
    }
    if (RES && issuer && res_pending) drain_wait(&sh.rfull[half], res_phase & 1);  // an abort left a load in flight
    if (S::STAGING && issuer) tma_store_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace blockgemm
}  // namespace b200
