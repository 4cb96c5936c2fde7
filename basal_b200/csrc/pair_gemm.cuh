// The block-scaled GEMM of the FP8-block and INT8-block formats on a CTA pair (tcgen05 cta_group::2), for bf16 / fp16
// outputs. The same arithmetic as block_gemm.cuh (per 128-deep slice: product in TMEM, times a_s * b_s, added into
// fp32 registers), with the work split so that less data crosses from L2 and the stores do not stall the promotion:
//
//   * a cluster of 2 CTAs computes a 256 x 256 output tile: each CTA loads its 128 rows of A and 128 of the 256
//     weight rows (B split along N), 32 KB a slice instead of 48 KB for a 128 x 256 tile per CTA; the pair's leader
//     issues one M = 256, N = 256 MMA that writes 128 rows into each CTA's TMEM. No load goes to more than one CTA.
//   * both CTAs' copies complete on the leader's `full` barrier; the leader's commits arrive on both CTAs' `empty`
//     (stage free) and `tfull` (accumulator complete) barriers; both CTAs' promotion warps arrive on the leader's
//     `tempty` (accumulator read) barrier.
//   * the epilogue writes the cast tile (and bias) into a 64 KB shared staging buffer in the 128-byte swizzle and
//     hands it to TMA stores (asynchronous; rows past M are clipped by the tensor map), so the promotion of the next
//     tile starts at once.
// Roles per CTA as in block_gemm.cuh: warp 0 producer, warp 1 MMA issuer (leader only), warp 2 TMEM, warps 4-11
// promotion and epilogue (setmaxnreg 40 / 232).
#pragma once
#include "block_gemm.cuh"

namespace b200 {
namespace pairgemm {

constexpr int BM = 128;                   // rows a CTA (256 a pair)
constexpr int BN = 256;                   // output columns of a pair tile
constexpr int BK = 128;                   // K bytes a stage
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;          // 16 KB
constexpr int B_BYTES = (BN / 2) * BK;    // 16 KB: this CTA's half of the weight rows
constexpr uint32_t PAIR_TX = 2 * (A_BYTES + B_BYTES);
constexpr int SUB_BYTES = BM * 128;       // one 64-column x 128-row sub-tile of 16-bit outputs
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr int NUM_EPI_WARPS = 8;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t REGS_LOW = 40, REGS_HIGH = 232;
constexpr uint32_t LAUNCH_REGS = (REGS_LOW * 128 + REGS_HIGH * 256) / NUM_THREADS;

struct Shared {
  uint8_t out[4][SUB_BYTES];  // staging of the 128 x 256 output block, 4 sub-tiles, 128-byte swizzle
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mdrain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t SMEM_BYTES = sizeof(Shared) + 1024;

struct Params {
  const float* s;    // [M, K/128]
  const float* ws;   // [N/128, K/128]
  const void* bias;  // [N] in the output type, or null
  int M, N, nkb, tiles_n, num_tiles;
};

__device__ __forceinline__ bool warp_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  unsigned fault) {
  const bool ok = mbar_wait_cluster(bar, parity, abort_flag, fault);
  return __all_sync(0xffffffffu, ok);
}

// Offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled sub-tile (the layout TMA reads with
// CU_TENSOR_MAP_SWIZZLE_128B).
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <bool INT8, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const Params p) {
  static_assert(OUT == BASAL200_BF16 || OUT == BASAL200_F16, "16-bit outputs (TMA-store epilogue)");
  using OutT = typename blockgemm::Store<OUT>::T;
  extern __shared__ uint8_t smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.tfull[b], 1);
      mbar_init(&sh.tempty[b], 2 * NUM_EPI_WARPS);
    }
    mbar_init(&sh.mdrain, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 2) tmem_alloc_pair(&sh.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any copy or arrive reaches them
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;
  const uint32_t full_leader = cluster_addr(smem_u32(&sh.full[0]), 0);
  const uint32_t tempty_leader = cluster_addr(smem_u32(&sh.tempty[0]), 0);

  if (warp < EPI_WARP0) regs_release<REGS_LOW>();
  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, filled = 0, last_phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < p.num_tiles; tile += npairs) {
        const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
        for (int kb = 0; kb < p.nkb; ++kb) {
          if (!mbar_wait_cluster(&sh.empty[stage], phase ^ 1, abort_flag, kFaultTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&sh.full[stage], PAIR_TX);
          tma_load_2d_pair(sh.a[stage], &tmA, full_leader + stage * 8, kb * BK, tm * 2 * BM + (int)rank * BM);
          tma_load_2d_pair(sh.b[stage], &tmB, full_leader + stage * 8, kb * BK, tn * BN + (int)rank * (BN / 2));
          filled |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        if (leader) {
          for (int s = 0; s < STAGES; ++s)
            if (filled & (1u << s)) blockgemm::drain_wait(&sh.full[s], (last_phase >> s) & 1);
        } else {  // the peer's copies complete on the leader's barriers: give them time to land
          const unsigned long long t0 = globaltimer();
          while (globaltimer() - t0 < 100000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the pair's leader) ----------------
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = INT8 ? idesc_dense(2, 1, 1, 2 * BM, BN) : idesc_dense(1, 0, 0, 2 * BM, BN);
      const uint32_t empty0 = cluster_addr(smem_u32(&sh.empty[0]), 0), empty1 = cluster_addr(smem_u32(&sh.empty[0]), 1);
      const uint32_t tfull0 = cluster_addr(smem_u32(&sh.tfull[0]), 0), tfull1 = cluster_addr(smem_u32(&sh.tfull[0]), 1);
      int stage = 0;
      uint32_t phase = 0, acc = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < p.num_tiles; tile += npairs) {
        for (int kb = 0; kb < p.nkb; ++kb) {
          const uint32_t buf = acc & 1, aph = (acc >> 1) & 1;
          if (!mbar_wait_cluster(&sh.tempty[buf], aph ^ 1, abort_flag, kFaultTimeoutMma) ||
              !mbar_wait_cluster(&sh.full[stage], phase, abort_flag, kFaultTimeoutMma)) {
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
              mma_i8_pair(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
            else
              mma_f8f6f4_pair(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
          }
          mma_commit_pair(empty0 + stage * 8);
          mma_commit_pair(empty1 + stage * 8);
          mma_commit_pair(tfull0 + buf * 8);
          mma_commit_pair(tfull1 + buf * 8);
          ++acc;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      mma_commit_pair(cluster_addr(smem_u32(&sh.mdrain), 0));
      blockgemm::drain_wait(&sh.mdrain, 0);
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- promotion and epilogue (both CTAs) ----------------
    regs_claim<REGS_HIGH>();
    const int ew = warp - EPI_WARP0;
    const int half = ew >> 2;   // which 128 columns of the 256-wide tile
    const int quad = warp & 3;  // the TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;  // row within this CTA's 128 rows
    const bool issuer = (ew & 3) == 0 && lane == 0;
    const int nkb = p.nkb;
    uint32_t acc_cnt = 0;
    bool ok = true;
    for (int tile = pair; tile < p.num_tiles; tile += npairs) {
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      const int row0 = tm * 2 * BM + (int)rank * BM;
      const int row = row0 + r;
      const int n0 = tn * BN + half * 128;
      const bool nvalid = n0 < p.N;
      const float* srow = p.s + (int64_t)min(row, p.M - 1) * nkb;
      const float* wsr = p.ws + (int64_t)min(n0 / 128, p.N / 128 - 1) * nkb;
      uint64_t acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0ull;
      float sa = __ldg(srow), sb = __ldg(wsr);
      for (int kb = 0; kb < nkb; ++kb) {
        const float sc = sa * sb;
        const uint64_t sc2 = pack_f2(sc, sc);
        if (kb + 1 < nkb) {
          sa = __ldg(srow + kb + 1);
          sb = __ldg(wsr + kb + 1);
        }
        const uint32_t buf = acc_cnt & 1, ph = (acc_cnt >> 1) & 1;
        if (!warp_wait_cluster(&sh.tfull[buf], ph, abort_flag, kFaultTimeoutEpilogue)) {
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
            if (lane == 0) mbar_arrive_remote(tempty_leader + buf * 8);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) ffma2p(acc[h * 32 + j], x[j], sc2);
        }
        ++acc_cnt;
      }
      // ---- epilogue: cast (+ bias) into the staging sub-tiles of this half, then TMA stores ----
      if (issuer) tma_store_wait_read();  // the previous tile's stores have read the staging
      ok = named_barrier_and(1 + half, 128, ok);  // the warpgroup agrees whether to go on
      if (!ok) break;
      const OutT* bias = (p.bias && nvalid) ? reinterpret_cast<const OutT*>(p.bias) + n0 : nullptr;
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // 16 chunks of 8 outputs
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_f2(acc[j * 4 + i]);
          v[2 * i] = f.x;
          v[2 * i + 1] = f.y;
        }
        OutT* dst = reinterpret_cast<OutT*>(sh.out[half * 2 + (j >> 3)] + sw128(r, j & 7));
        blockgemm::Store<OUT>::vec8(dst, v, bias ? bias + j * 8 : nullptr);
      }
      fence_proxy_async();
      named_barrier(1 + half, 128);
      if (issuer) {
        if (nvalid && row0 < p.M) {
          tma_store_2d(&tmC, sh.out[half * 2], n0, row0);
          tma_store_2d(&tmC, sh.out[half * 2 + 1], n0 + 64, row0);
        }
        tma_store_commit();
      }
    }
    if (issuer) tma_store_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its pair may still signal its barriers
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace pairgemm
}  // namespace b200
