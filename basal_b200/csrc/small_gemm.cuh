// The block-scaled GEMM of the FP8-block and INT8-block formats for few rows (M <= 64: decode steps, short chunks),
// where the weights are nearly all of the bytes and the GEMM is bound by how fast the weights stream from HBM.
//
// The same arithmetic as block_gemm.cuh, element for element: per 128-deep slice kb the exact product of the codes
// (tcgen05.mma, kind::f8f6f4 -> f32 or kind::i8 -> s32), then acc = fma(product, a_s * b_s, acc) in slice order from
// zero, a_s * b_s rounded once. So a row's output is bit-identical whichever kernel computes it and whatever the other
// rows are, as the reference requires (basal/blockquant.py:14-16, tests/test_fp8block.py:134-148): the chain is never
// reassociated (the split variant at the end of this file spreads the slices' products over the SMs, then runs the same
// chain in order).
//
// Operands swapped: a tile is 128 weight rows (the MMA's M) x NT token rows (the MMA's N: 32 or 64, the rows past M
// read as zeros). The products of two codes are exact and the MMA reduces along K either way, so the swap changes no
// bit of a slice's product.
//
// What bounds it, measured on B200: one SM fetches a 16 KB slice from HBM about every 0.3-0.4 us (the requests one SM
// keeps in flight cover about 50 KB, whatever the ring depth), and one thread issuing a slice's 4 MMAs and their
// commits, or one warp testing a barrier and loading a slice's product, spends hundreds of cycles in issue latency,
// which few tokens cannot hide. (Spreading a tile's loads over a cluster, with loader CTAs pushing slices into the
// leader's ring through distributed shared memory, was measured slower: the go-ahead/push round trip per stage costs
// about as much as the DRAM latency it hides.) So one CTA streams one 128-row weight tile through its whole K, and:
//   * three MMA issuers (warps 1-3; slice kb by warp 1 + kb % 3) overlap their issue latency; each owns every third
//     stage of the ring (9 stages for NT = 32, 6 for NT = 64) and its column block of the two TMEM product groups, so
//     every barrier's phases are produced and awaited in one thread's program order (a parity wait only tells the
//     current phase from the one before);
//   * the promotion takes the products three slices at a time (one barrier, three TMEM loads, one wait, one release),
//     with every a_s * b_s of the tile computed into shared memory before the first slice; 32 tokens a warp (4 warps
//     for NT = 32, 8 for NT = 64), thread = weight row; at the end the cast (and bias) and the stores, each token's 128
//     outputs consecutive.
#pragma once
#include <type_traits>

#include "block_gemm.cuh"

namespace b200 {
namespace smallgemm {

constexpr int BW = 128;            // weight rows a tile (the MMA's M)
constexpr int BK = 128;            // K bytes a slice
constexpr int W_BYTES = BW * BK;   // 16 KB
constexpr int MMA_WARPS = 3;       // warps 1-3 issue the MMAs
constexpr int GROUP = MMA_WARPS;   // slices a product group (one per issuer)
constexpr int GSLOTS = 2;          // product groups in TMEM

constexpr int EPI_WARP0 = 4;
constexpr int MAX_ROWS = 64;       // rows served by this kernel
constexpr int MAX_KB = 64;         // K <= 8192 (all scales of a tile in shared memory)

template <int NT>
struct Cfg {
  static constexpr int T_BYTES = NT * BK;
  static constexpr int STAGE_BYTES = W_BYTES + T_BYTES;  // weights then tokens
  static constexpr int STAGES = NT == 32 ? 9 : 6;        // a multiple of MMA_WARPS (stage ownership)
  static_assert(STAGES % MMA_WARPS == 0, "stage ownership");
  static constexpr int EPI_WARPS = NT / 32 * 4;          // 32 tokens a warp
  static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
  static constexpr uint32_t TMEM_COLS = GSLOTS * GROUP * NT <= 256 ? 256 : 512;  // a power of two
};

template <int NT>
struct Smem {
  static constexpr int STAGES = Cfg<NT>::STAGES;
  uint8_t stage[STAGES][Cfg<NT>::STAGE_BYTES];  // [weights 128 x 128][tokens NT x 128], 128-byte swizzle each
  float sc[MAX_KB][NT];                          // a_s[token, kb] * b_s[tile, kb]
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t gfull[GSLOTS];
  uint64_t gempty[GSLOTS];
  uint64_t mdrain;
  uint32_t tmem_base;
  int abort;
};
template <int NT>
constexpr size_t smem_bytes() {
  return sizeof(Smem<NT>) + 1024;
}

struct Params {
  const float* s;    // [M, K/128] activation scales
  const float* ws;   // [N/128, K/128] weight scales
  const void* bias;  // [N] in the output type, or null
  void* cs[blockgemm::kMaxPeers];  // the output buffers: [M, ldc] each, this GEMM's N columns from col_off (one, or
  int npeers;                      // every rank's for a column-parallel linear gathered by the stores)
  int64_t ldc;
  int col_off;
  int M, N, nkb;
  const uint32_t* gate = nullptr;  // gathered linear: this rank's peer-barrier status word (or null); non-zero = store nothing
};

// One bf16 / f16 / f32 output, with the bias added to the cast value and rounded again (as blockgemm::Store).
template <int OUT>
__device__ __forceinline__ void store1(void* c, int64_t idx, float v, const void* bias, int n) {
  if (OUT == BASAL200_BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    if (bias)
      h = __float2bfloat16_rn(
          __fadd_rn(__bfloat162float(h), __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n])));
    static_cast<__nv_bfloat16*>(c)[idx] = h;
  } else if (OUT == BASAL200_F16) {
    __half h = __float2half_rn(v);
    if (bias) h = __float2half_rn(__fadd_rn(__half2float(h), __half2float(static_cast<const __half*>(bias)[n])));
    static_cast<__half*>(c)[idx] = h;
  } else {
    if (bias) v = __fadd_rn(v, static_cast<const float*>(bias)[n]);
    static_cast<float*>(c)[idx] = v;
  }
}

// acc (16 packed pairs: this warp's 32 tokens) += product x scale, scale = a_s * b_s of the token (the large-M kernel's
// rounding: one product, then one fma per element).
template <bool INT8>
__device__ __forceinline__ void promote32(uint64_t (&acc)[16], const uint32_t (&x)[32], const float* sc) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    uint32_t lo = x[j], hi = x[j + 1];
    if (INT8) {
      lo = __float_as_uint(__int2float_rn((int)lo));
      hi = __float_as_uint(__int2float_rn((int)hi));
    }
    ffma2p(acc[j / 2], pack_u2(lo, hi), *reinterpret_cast<const uint64_t*>(sc + j));
  }
}

template <bool INT8, int OUT, int NT>
__global__ void __launch_bounds__(Cfg<NT>::THREADS, 1)
    small_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmT,
                      const Params p) {
  using S = Smem<NT>;
  using C = Cfg<NT>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  S& sh = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();
  const int nkb = p.nkb;
  const int ngroups = (nkb + GROUP - 1) / GROUP;
  const int tile = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int g = 0; g < GSLOTS; ++g) {
      mbar_init(&sh.gfull[g], MMA_WARPS);
      mbar_init(&sh.gempty[g], C::EPI_WARPS);
    }
    mbar_init(&sh.mdrain, MMA_WARPS);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmT);
  }
  if (warp == 2) tmem_alloc(&sh.tmem_base, C::TMEM_COLS);
  pdl_launch();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  {
    if (warp == 0) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        uint32_t filled = 0, last_phase = 0;
        // the weights of the first ring of slices load while the kernel before this one finishes (no kernel that
        // lets its successor start early writes weights); the tokens, an earlier kernel's output, after pdl_wait
        const int pre = nkb < STAGES ? nkb : STAGES;
        for (int kb = 0; kb < pre; ++kb) {
          mbar_arrive_expect_tx(&sh.full[kb], C::STAGE_BYTES);
          tma_load_2d(sh.stage[kb], &tmW, &sh.full[kb], kb * BK, tile * BW);
          filled |= 1u << kb;
        }
        pdl_wait();
        for (int kb = 0; kb < pre; ++kb) tma_load_2d(sh.stage[kb] + W_BYTES, &tmT, &sh.full[kb], kb * BK, 0);
        for (int kb = pre; kb < nkb; ++kb) {
          const int stage = kb % STAGES;
          const uint32_t phase = (uint32_t)(kb / STAGES) & 1;
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, abort_flag, kFaultTimeoutProducer)) break;
          mbar_arrive_expect_tx(&sh.full[stage], C::STAGE_BYTES);
          tma_load_2d(sh.stage[stage], &tmW, &sh.full[stage], kb * BK, tile * BW);
          tma_load_2d(sh.stage[stage] + W_BYTES, &tmT, &sh.full[stage], kb * BK, 0);
          filled |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
        }
        if (*abort_flag) {  // let the copies already issued land
          for (int s = 0; s < STAGES; ++s)
            if (filled & (1u << s)) blockgemm::drain_wait(&sh.full[s], (last_phase >> s) & 1);
        }
      }
    } else if (warp < EPI_WARP0) {
      // ---------------- MMA issuers: warp 1 + i issues slice 3g + i of every group g ----------------
      if (lane == 0) {
        constexpr uint32_t idesc = INT8 ? idesc_dense(2, 1, 1, BW, NT) : idesc_dense(1, 0, 0, BW, NT);
        const int i = warp - 1;
        for (int g = 0; g < ngroups; ++g) {
          const int slot = g % GSLOTS;
          // the group's TMEM block is free (its previous group was read); an issuer without a slice in the last
          // group still waits and commits, so every group's barrier phase gets its three arrivals in order
          if (!mbar_wait(&sh.gempty[slot], ((uint32_t)(g / GSLOTS) & 1) ^ 1, abort_flag, kFaultTimeoutMma)) break;
          const int kb = g * GROUP + i;
          if (kb < nkb) {
            const int stage = kb % STAGES;
            if (!mbar_wait(&sh.full[stage], (uint32_t)(kb / STAGES) & 1, abort_flag, kFaultTimeoutMma)) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)((slot * GROUP + i) * NT);
            const uint64_t ad = desc_sw128(smem_u32(sh.stage[stage]));
            const uint64_t bd = desc_sw128(smem_u32(sh.stage[stage] + W_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 32; ++k) {
              if (INT8)
                mma_i8(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
              else
                mma_f8f6f4(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
            }
            mma_commit(&sh.empty[stage]);
          }
          mma_commit(&sh.gfull[slot]);
        }
        // every MMA this thread issued has finished before TMEM and shared memory are released
        mma_commit(&sh.mdrain);
        blockgemm::drain_wait(&sh.mdrain, 0);
      }
    } else {
      // ---------------- promotion and epilogue ----------------
      const int ew = warp - EPI_WARP0;
      const int quad = warp & 3;       // TMEM lane quadrant: weight rows quad * 32 ..
      const int half = ew >> 2;        // which 32 of the NT tokens
      const int t = quad * 32 + lane;  // weight row of the tile
      const int et = ew * 32 + lane;   // index among the promotion threads
      constexpr int ETHREADS = C::EPI_WARPS * 32;
      const uint32_t tcol = tmem + ((uint32_t)(quad * 32) << 16) + half * 32;
      // every a_s * b_s of the tile, while the first slices load (token j's scales are contiguous); the scales and
      // this thread's stores come after the kernels before this one
      pdl_wait();
      const int npeers = blockgemm::stored_peers(p.npeers, p.gate);
      for (int idx = et; idx < NT * nkb; idx += ETHREADS) {
        const int j = idx / nkb, kb = idx - j * nkb;
        sh.sc[kb][j] = j < p.M ? __ldg(p.s + (int64_t)j * nkb + kb) * __ldg(p.ws + (int64_t)tile * nkb + kb) : 0.f;
      }
      named_barrier(1, ETHREADS);
      uint64_t acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0ull;
      bool ok = true;
      for (int g = 0; ok && g < ngroups; ++g) {
        const int slot = g % GSLOTS;
        if (!blockgemm::warp_wait(&sh.gfull[slot], (uint32_t)(g / GSLOTS) & 1, abort_flag, kFaultTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n = nkb - g * GROUP < GROUP ? nkb - g * GROUP : GROUP;  // slices in this group
        uint32_t x0[32], x1[32], x2[32];
        const uint32_t base = tcol + (uint32_t)(slot * GROUP * NT);
        tmem_ld32_issue(base, x0);
        if (n > 1) tmem_ld32_issue(base + NT, x1);
        if (n > 2) tmem_ld32_issue(base + 2 * NT, x2);
        tmem_ld_wait32(x0);  // one wait covers every load in flight; the other two name their registers
        tmem_ld_wait32(x1);
        tmem_ld_wait32(x2);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.gempty[slot]);
        const int kb = g * GROUP;
        promote32<INT8>(acc, x0, &sh.sc[kb][half * 32]);
        if (n > 1) promote32<INT8>(acc, x1, &sh.sc[kb + 1][half * 32]);
        if (n > 2) promote32<INT8>(acc, x2, &sh.sc[kb + 2][half * 32]);
      }
      if (ok) {
        // cast (+ bias) and store: token j's outputs of this tile are 128 consecutive values
        const int n = tile * BW + t;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 v = unpack_f2(acc[j / 2]);
          const int tok = half * 32 + j;
          for (int r = 0; r < npeers; ++r) {
            if (tok < p.M) store1<OUT>(p.cs[r], (int64_t)tok * p.ldc + p.col_off + n, v.x, p.bias, n);
            if (tok + 1 < p.M) store1<OUT>(p.cs[r], (int64_t)(tok + 1) * p.ldc + p.col_off + n, v.y, p.bias, n);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------------------------------------------
// The same GEMM with the slices spread over every SM, for weights of fewer 128-row tiles than the GPU has SMs (N <
// 19,000 or so): the kernel above puts one CTA on each tile, so at N = 2048 16 SMs stream the weights and the rest
// idle. Here the (tile, slice) units are dealt out in contiguous runs to min(#SMs, units) CTAs, each of which writes
// the raw 128-deep product of each of its units (fp32; INT8's s32 products, below 2^21, converted exactly) to a
// workspace; a second kernel then runs, per output, the same chain acc = fma(product_kb, a_s * b_s, acc) in slice
// order from zero as both other kernels. So a row's bits still do not depend on the kernel or on the other rows.
// The products cost 4 bytes per (token, output, slice) of workspace traffic, which stays in L2 at these sizes.
// ---------------------------------------------------------------------------------------------------------------
template <int NT>
struct SplitCfg {
  static constexpr int STAGE_BYTES = W_BYTES + NT * BK;
  static constexpr int STAGES = NT == 32 ? 9 : 6;  // multiples of MMA_WARPS: each stage and each TMEM slot is served
  static constexpr int TSLOTS = NT == 32 ? 15 : 6;  // by one issuer, so its barrier phases come in program order
  static_assert(STAGES % MMA_WARPS == 0 && TSLOTS % MMA_WARPS == 0, "stage / slot ownership");
  static_assert(TSLOTS * NT <= 512, "TMEM columns");
  static constexpr int EPI_WARPS = NT / 32 * 4;
  static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
  static constexpr int QUANT_WARPS = NT == 32 ? 8 : 4;  // the fused linear's activation quantisers, after the readout
                                                        // warps (as many as the registers of the launch allow)
  static constexpr uint32_t TMEM_COLS = 512;
};

template <int NT>
struct SplitSmem {
  static constexpr int STAGES = SplitCfg<NT>::STAGES;
  static constexpr int TSLOTS = SplitCfg<NT>::TSLOTS;
  uint8_t stage[STAGES][SplitCfg<NT>::STAGE_BYTES];  // [weights 128 x 128][tokens NT x 128], 128-byte swizzle each
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[TSLOTS];
  uint64_t tempty[TSLOTS];
  uint64_t mdrain;
  uint32_t tmem_base;
  int abort;
};
template <int NT>
constexpr size_t split_smem_bytes() {
  return sizeof(SplitSmem<NT>) + 1024;
}

struct SplitParams {
  float* prod;    // [N/128][nkb][M][128] fp32: unit (tile, kb)'s product of token j and weight row r
  int64_t units;  // (N / 128) * nkb
  int M, nkb;
  const void* x;  // fused linear only: the activations [M, nkb * 128] (16-bit), quantised here instead of loaded as
  float* s;       // codes; their scales [M, nkb] are written to s for the second kernel
};

// Workspace bytes of the split kernels for M tokens, N outputs and nkb slices.
__host__ __device__ constexpr int64_t split_prod_bytes(int64_t M, int64_t N, int64_t nkb) { return M * N * nkb * 4; }

// TX = void: the token codes of a unit come by TMA (tmT). TX = bf16 / f16: the fused linear; QUANT_WARPS more warps
// quantise the activations slice by slice (one half-warp a token: the next slice's 16-byte loads issued while this one
// is quantised, amax by shuffles, blockquant's codes by block_codes8, exactly as act_quant_block_kernel) and write the
// codes into each unit's stage where the TMA would have put them, in the same 128-byte swizzle.
template <int NT, typename TX>
constexpr int split_threads() {
  return SplitCfg<NT>::THREADS + (std::is_void<TX>::value ? 0 : SplitCfg<NT>::QUANT_WARPS * 32);
}

template <bool INT8, int NT, typename TX>
__global__ void __launch_bounds__(split_threads<NT, TX>(), 1)
    split_products_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmT,
                          const SplitParams p) {
  using S = SplitSmem<NT>;
  using C = SplitCfg<NT>;
  constexpr bool QUANT = !std::is_void<TX>::value;
  constexpr int STAGES = C::STAGES;
  constexpr int TSLOTS = C::TSLOTS;
  constexpr uint32_t LOAD_BYTES = QUANT ? W_BYTES : C::STAGE_BYTES;  // TMA bytes a stage
  extern __shared__ uint8_t smem_raw[];
  S& sh = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();
  const int nkb = p.nkb;
  const int tiles = (int)(p.units / nkb);
  // this CTA's run of units [u0, u0 + nu). TMA tokens: unit u is slice u % nkb of weight tile u / nkb (a run walks
  // along K). Fused quantiser: slice u / tiles of tile u % tiles (a run walks across tiles at one or two slices, so
  // each slice is quantised once a CTA, not once a unit).
  const int64_t u0 = (int64_t)blockIdx.x * p.units / gridDim.x;
  const int nu = (int)((int64_t)(blockIdx.x + 1) * p.units / gridDim.x - u0);
  auto unit_kb = [&](int64_t u) { return QUANT ? (int)(u / tiles) : (int)(u % nkb); };
  auto unit_tile = [&](int64_t u) { return QUANT ? (int)(u % tiles) : (int)(u / nkb); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], QUANT ? 1 + C::QUANT_WARPS : 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int t = 0; t < TSLOTS; ++t) {
      mbar_init(&sh.tfull[t], 1);
      mbar_init(&sh.tempty[t], C::EPI_WARPS);
    }
    mbar_init(&sh.mdrain, MMA_WARPS);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (QUANT) {  // token rows past M stay zero in every stage (the quantisers write rows < M only)
    for (int i = threadIdx.x; i < STAGES * NT * BK / 16; i += blockDim.x) {
      const int st = i / (NT * BK / 16), o = i - st * (NT * BK / 16);
      reinterpret_cast<uint4*>(sh.stage[st] + W_BYTES)[o] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async();  // visible to the tensor cores' reads
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmT);
  }
  if (warp == 2) tmem_alloc(&sh.tmem_base, C::TMEM_COLS);
  pdl_launch();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t filled = 0, last_phase = 0;
      // weights of the first ring of units before pdl_wait (no kernel that lets its successor start early writes
      // weights); the tokens, an earlier kernel's output, after it
      const int pre = nu < STAGES ? nu : STAGES;
      for (int j = 0; j < pre; ++j) {
        const int64_t u = u0 + j;
        mbar_arrive_expect_tx(&sh.full[j], LOAD_BYTES);
        tma_load_2d(sh.stage[j], &tmW, &sh.full[j], unit_kb(u) * BK, unit_tile(u) * BW);
        filled |= 1u << j;
      }
      if (!QUANT) {
        pdl_wait();
        for (int j = 0; j < pre; ++j)
          tma_load_2d(sh.stage[j] + W_BYTES, &tmT, &sh.full[j], unit_kb(u0 + j) * BK, 0);
      }
      for (int j = pre; j < nu; ++j) {
        const int stage = j % STAGES;
        const uint32_t phase = (uint32_t)(j / STAGES) & 1;
        if (!mbar_wait(&sh.empty[stage], phase ^ 1, abort_flag, kFaultTimeoutProducer)) break;
        const int64_t u = u0 + j;
        mbar_arrive_expect_tx(&sh.full[stage], LOAD_BYTES);
        tma_load_2d(sh.stage[stage], &tmW, &sh.full[stage], unit_kb(u) * BK, unit_tile(u) * BW);
        if (!QUANT) tma_load_2d(sh.stage[stage] + W_BYTES, &tmT, &sh.full[stage], unit_kb(u) * BK, 0);
        filled |= 1u << stage;
        last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
      }
      if (*abort_flag) {  // let the copies already issued land
        for (int s = 0; s < STAGES; ++s)
          if (filled & (1u << s)) blockgemm::drain_wait(&sh.full[s], (last_phase >> s) & 1);
      }
    }
  } else if (warp < EPI_WARP0) {
    // ---------------- MMA issuers: warp 1 + i issues units i, i + 3, ... ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = INT8 ? idesc_dense(2, 1, 1, BW, NT) : idesc_dense(1, 0, 0, BW, NT);
      const int i = warp - 1;
      for (int j = i; j < nu; j += MMA_WARPS) {
        const int slot = j % TSLOTS;
        if (!mbar_wait(&sh.tempty[slot], ((uint32_t)(j / TSLOTS) & 1) ^ 1, abort_flag, kFaultTimeoutMma)) break;
        const int stage = j % STAGES;
        if (!mbar_wait(&sh.full[stage], (uint32_t)(j / STAGES) & 1, abort_flag, kFaultTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(slot * NT);
        const uint64_t ad = desc_sw128(smem_u32(sh.stage[stage]));
        const uint64_t bd = desc_sw128(smem_u32(sh.stage[stage] + W_BYTES));
#pragma unroll
        for (int k = 0; k < BK / 32; ++k) {
          if (INT8)
            mma_i8(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
          else
            mma_f8f6f4(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
        }
        mma_commit(&sh.empty[stage]);
        mma_commit(&sh.tfull[slot]);
      }
      // every MMA this thread issued has finished before TMEM and shared memory are released
      mma_commit(&sh.mdrain);
      blockgemm::drain_wait(&sh.mdrain, 0);
    }
  } else if (QUANT && warp >= EPI_WARP0 + C::EPI_WARPS) {
    // ------- activation quantisers (fused linear): token t = pass * 2 * QUANT_WARPS + qw * 2 + half -------
    if constexpr (QUANT) {
      constexpr int TPP = 2 * C::QUANT_WARPS;  // tokens a pass (a half-warp each)
      constexpr int PASSES = NT / TPP;
      constexpr int W = sizeof(TX) / 2;  // 16-byte words of a lane's 8 values (one: 16-bit activations)
      static_assert(W == 1, "the fused quantiser takes 16-bit activations");
      constexpr float kQmax = INT8 ? 127.0f : 448.0f;
      const int qw = warp - EPI_WARP0 - C::EPI_WARPS;
      const int hf = lane >> 4, l16 = lane & 15;
      const TX* x = static_cast<const TX*>(p.x);
      const int64_t ldx = (int64_t)nkb * BK;
      uint4 raw[PASSES][1];  // the activations of the next slice to quantise, loaded ahead
      uint2 codes[PASSES];   // the codes of slice kb_cur
      auto load_slice = [&](int kb) {
#pragma unroll
        for (int ps = 0; ps < PASSES; ++ps) {
          const int t = ps * TPP + qw * 2 + hf;
          if (t < p.M)
            raw_load8(x + t * ldx + kb * BK + l16 * 8, raw[ps]);
          else
            raw[ps][0] = make_uint4(0u, 0u, 0u, 0u);
        }
      };
      const int kb_last = nu > 0 ? unit_kb(u0 + nu - 1) : 0;
      int kb_cur = -1;
      pdl_wait();  // the activations are an earlier kernel's output; the scales go where it may still read
      if (nu > 0) load_slice(unit_kb(u0));
      for (int j = 0; j < nu; ++j) {
        const int kb = unit_kb(u0 + j);
        if (kb != kb_cur) {  // a new slice: quantise the loaded activations, then load the next slice's
#pragma unroll
          for (int ps = 0; ps < PASSES; ++ps) {
            if (ps * TPP >= p.M) break;  // no token of this pass is real (the same for every lane)
            const int t = ps * TPP + qw * 2 + hf;
            float v[8];
            unpack8(raw[ps], x, v);
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), kQmax);
            codes[ps] = block_codes8<INT8>(v, sc);
            if (t < p.M && l16 == 0) p.s[(int64_t)t * nkb + kb] = sc;  // every CTA with slice kb: the same value
          }
          kb_cur = kb;
          if (kb + 1 <= kb_last) load_slice(kb + 1);
        }
        const int stage = j % STAGES;
        if (j >= STAGES &&
            !blockgemm::warp_wait(&sh.empty[stage], ((uint32_t)(j / STAGES) & 1) ^ 1, abort_flag,
                                  kFaultTimeoutProducer))
          break;
        uint8_t* tok = sh.stage[stage] + W_BYTES;
#pragma unroll
        for (int ps = 0; ps < PASSES; ++ps) {
          const int t = ps * TPP + qw * 2 + hf;
          if (t < p.M) *reinterpret_cast<uint2*>(tok + blockgemm::sw128(t, l16 >> 1) + (l16 & 1) * 8) = codes[ps];
        }
        fence_proxy_async();  // the codes, visible to the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.full[stage]);
      }
    }
  } else {
    // ---------------- product readout: thread = weight row, 32 tokens a warp ----------------
    const int ew = warp - EPI_WARP0;
    const int quad = warp & 3;       // TMEM lane quadrant: weight rows quad * 32 ..
    const int half = ew >> 2;        // which 32 of the NT tokens
    const int t = quad * 32 + lane;  // weight row of the tile
    const int ntok = p.M - half * 32 < 32 ? p.M - half * 32 : 32;  // this warp's real tokens (may be <= 0)
    const uint32_t tcol = tmem + ((uint32_t)(quad * 32) << 16) + half * 32;
    pdl_wait();  // the workspace may still be read by the kernel before this one
    for (int j = 0; j < nu; ++j) {
      const int slot = j % TSLOTS;
      if (!blockgemm::warp_wait(&sh.tfull[slot], (uint32_t)(j / TSLOTS) & 1, abort_flag, kFaultTimeoutEpilogue))
        break;
      tc_fence_after();
      uint32_t x[32];
      tmem_ld32_issue(tcol + (uint32_t)(slot * NT), x);
      tmem_ld_wait32(x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty[slot]);
      const int64_t u = u0 + j;
      float* dst = p.prod + (((int64_t)unit_tile(u) * nkb + unit_kb(u)) * p.M + half * 32) * BW + t;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (jj < ntok) __stcg(dst + (int64_t)jj * BW, INT8 ? __int2float_rn((int)x[jj]) : __uint_as_float(x[jj]));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Second kernel of the split GEMM: a CTA per (token, weight tile), thread = weight row. a_s * b_s of the token and tile
// for every slice go to shared memory first; then every slice's product is loaded at once (one L2 round trip, not one
// per slice) and summed in slice order, acc = fma(product, a_s * b_s, acc) from zero; then the cast (+ bias) and the
// stores.
constexpr int REDUCE_THREADS = BW;

template <int OUT>
__global__ void __launch_bounds__(REDUCE_THREADS)
    split_reduce_kernel(const float* __restrict__ prod, const Params p) {
  __shared__ float sc[MAX_KB];
  pdl_launch();
  pdl_wait();  // the products kernel has completed and its stores are visible
  const int tile = blockIdx.x;
  const int tok = blockIdx.y;
  const int row = threadIdx.x;
  const int nkb = p.nkb;
  if (row < nkb) sc[row] = __fmul_rn(__ldg(p.s + (int64_t)tok * nkb + row), __ldg(p.ws + (int64_t)tile * nkb + row));
  const int64_t kstride = (int64_t)p.M * BW;
  const float* src = prod + ((int64_t)tile * nkb * p.M + tok) * BW + row;  // + kb * kstride
  float pv[MAX_KB];
#pragma unroll
  for (int kb = 0; kb < MAX_KB; ++kb)
    if (kb < nkb) pv[kb] = __ldcg(src + kb * kstride);
  __syncthreads();
  float acc = 0.f;
#pragma unroll
  for (int kb = 0; kb < MAX_KB; ++kb)
    if (kb < nkb) acc = __fmaf_rn(pv[kb], sc[kb], acc);
  const int n = tile * BW + row;
  const int npeers = blockgemm::stored_peers(p.npeers, p.gate);
#pragma unroll
  for (int r = 0; r < blockgemm::kMaxPeers; ++r)  // constant indices keep the parameter block out of local memory
    if (r < npeers) store1<OUT>(p.cs[r], (int64_t)tok * p.ldc + p.col_off + n, acc, p.bias, n);
}

}  // namespace smallgemm
}  // namespace b200
