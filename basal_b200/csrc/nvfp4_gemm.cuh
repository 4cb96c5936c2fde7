// The NVFP4 GEMM on sm_100a (replaces cuBLAS's block-scaled FP4 GEMM behind F.scaled_mm, basal/nvfp4.py:167-180):
//
//   Y[m, n] = alpha * sum_k (e2m1 A[m, k] * sA[m, k / 16]) * (e2m1 B[n, k] * sB[n, k / 16])
//
// with the e4m3 block scales applied by the tensor core itself (tcgen05.mma kind::mxf4nvf4, scale_vec::4X, K = 64
// an instruction). A [Mp, K/2] and B [N, K/2] are packed e2m1 (even feature in the low nibble), K-major. The scales
// are consumed as the reference stores them, in the 128 x 4 tile swizzle (512 bytes for 128 rows x 64 features):
// that tile, moved into TMEM by tcgen05.cp's 32x128b.warpx4 shape, is the layout the MMA reads (lane l, column c,
// byte j = scale of row 32 c + l % 32, feature group j); the 256 rows of a B tile take 8 columns, the first 128 rows
// in the first 4. Persistent CTAs walk 128 x 256 output tiles:
//   warp 0       producer: TMA of A / B (256 features = 128 bytes a stage, 128-byte swizzle) into a 4-stage ring and
//                plain bulk copies of the next step's 4 + 8 scale tiles into a 5-slot ring
//   warps 2, 3   scale issuers: tcgen05.cp of the stage's scale tiles to its TMEM columns (warp 2 those of A and of
//                the B tile's first 128 rows, warp 3 the second 128 rows), then a commit (sfready)
//   warp 1       MMA issuer: 4 MMAs of 128 x 256 x 64 a stage once its scales are in TMEM, commit
//   warps 4-19   epilogue: tcgen05.ld of 32 rows x 64 columns a warp, release of the accumulator, times alpha,
//                (+ bias), cast, a warp transpose of 16-byte chunks, stores of whole 128-byte row segments
// The tcgen05 instructions cost the issuing thread about as long to issue as a 128 x 128 x 64 MMA takes to run: a
// 128 x 128 tile whose one thread issued a stage's 8 copies and 4 MMAs ran at 285 us (M = 8192, N = 12288,
// K = 2048), 177 / 180 us with either half switched off. N = 256 halves the MMAs per product and the copies are
// spread over two threads. A step's scales are loaded one step ahead of its operands, into a ring one slot deeper than
// the operands', so that they are in TMEM before the operands land (the operand ring's round trip was load latency +
// copies + MMA issue; now it is load latency + MMA issue). The accumulator's 256 columns and 5 slots x 48 scale
// columns fill TMEM, so there is one accumulator: the epilogue reads it out to registers and releases it before it
// stores.
#pragma once
#include "block_gemm.cuh"

namespace b200 {
namespace fp4gemm {

constexpr int BM = 128;
constexpr int BKB = 128;  // bytes of K per stage (256 e2m1 values = 4 scale tiles)
constexpr int A_BYTES = BM * BKB;
constexpr int SF_BYTES = 4 * 512;  // 4 scale tiles of 128 rows
constexpr int NUM_EPI_WARPS = 16;
constexpr int EPI_WARP0 = 4;
constexpr int NUM_THREADS = (EPI_WARP0 + NUM_EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t SFA_COLS = 16;  // 4 chunks x 4 columns

// Tile width: BN = 256 (the rule), or 128 when 256-wide tiles would leave SMs idle (few rows): then a CTA streams
// 128 weight rows, and the smaller stages make room for a deeper ring (the bytes in flight that bound a few-rows
// GEMM). The arithmetic of an output element is the same in both.
template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;  // operand (A / B) ring
  static constexpr int SF_SLOTS = STAGES + 1;       // scale ring: a step's scales come one step ahead of its operands
  static constexpr int B_BYTES = BN * BKB;
  static constexpr int BHALVES = BN / 128;          // 128-row scale tiles of a B tile
  static constexpr uint32_t SF_COL0 = BN;           // scale columns after the accumulator
  static constexpr uint32_t SF_COLS_PER_STAGE = SFA_COLS + BN / 8;  // + 4 chunks x BN / 32 columns of B
  static constexpr int EPI_COLS = BN / 4;           // accumulator columns an epilogue warp reads
  static_assert(SF_COL0 + SF_SLOTS * SF_COLS_PER_STAGE <= TMEM_COLS, "TMEM budget");
  struct Shared {
    uint8_t a[STAGES][A_BYTES];
    uint8_t b[STAGES][B_BYTES];
    uint8_t sfa[SF_SLOTS][SF_BYTES];
    uint8_t sfb[SF_SLOTS][BHALVES][SF_BYTES];  // the B tile's 128-row halves
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t sffull[SF_SLOTS];
    uint64_t sfready[SF_SLOTS];
    uint64_t tfull;
    uint64_t tempty;
    uint64_t mdrain;
    uint32_t tmem_base;
    int abort;
  };
  static constexpr size_t SMEM_BYTES = sizeof(Shared) + 1024;
  static_assert(SMEM_BYTES <= 232448, "227 KB of shared memory a CTA");
};

struct Params {
  const uint8_t* sa;   // swizzled scales of A: Mp/128 x (K/64) tiles
  const uint8_t* sb;   // of B: ceil(N/128) x (K/64) tiles
  const float* alpha;  // [1]
  const void* bias;    // [N] output type, or null
  void* y;             // [M, N]
  int M, N, nchunk, nkb, tiles_n, num_tiles, nblk_b;  // nblk_b = ceil(N / 128)
};

template <int OUT, int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const Params p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES, SF_SLOTS = C::SF_SLOTS, B_BYTES = C::B_BYTES;
  constexpr uint32_t SF_COL0 = C::SF_COL0, SF_COLS_PER_STAGE = C::SF_COLS_PER_STAGE;
  using Shared = typename C::Shared;
  extern __shared__ uint8_t smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int s = 0; s < SF_SLOTS; ++s) {
      mbar_init(&sh.sffull[s], 1);
      mbar_init(&sh.sfready[s], 2);  // the two scale issuers
    }
    mbar_init(&sh.tfull, 1);
    mbar_init(&sh.tempty, NUM_EPI_WARPS);
    mbar_init(&sh.mdrain, 3);  // the MMA issuer and the two scale issuers
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) tmem_alloc(&sh.tmem_base, TMEM_COLS);
  pdl_launch();
  pdl_wait();  // the set-up above ran while the kernel before this one finished
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;
  const int64_t c4 = p.nchunk;  // scale tiles per 128-row block (K / 64)

  if (warp == 0) {
    if (lane == 0) {
      // step g = the g-th (tile, k-block) of this CTA: its operands go to stage g % STAGES, its scales (loaded one
      // step earlier, after the wait on `empty` that frees step g - STAGES's slots) to slot g % SF_SLOTS
      int stage = 0, slot = 0, sf_tile = blockIdx.x, sf_kb = 0;
      uint32_t phase = 0, sf_phase = 0, filled = 0, last_phase = 0, sf_filled = 0, sf_last = 0;
      auto load_scales = [&]() {
        if (sf_tile >= p.num_tiles) return;
        const int tm = sf_tile / p.tiles_n, tn = sf_tile - tm * p.tiles_n;
        const int64_t bb = (int64_t)tn * C::BHALVES;  // the tile's first 128-row block of B
        const bool b_hi = C::BHALVES == 2 && bb + 1 < p.nblk_b;  // its second 128 rows exist
        const int nch = min(4, p.nchunk - sf_kb * 4);
        mbar_arrive_expect_tx(&sh.sffull[slot], (b_hi ? 3 : 2) * nch * 512);
        bulk_load(sh.sfa[slot], p.sa + ((int64_t)tm * c4 + sf_kb * 4) * 512, nch * 512, &sh.sffull[slot]);
        bulk_load(sh.sfb[slot][0], p.sb + (bb * c4 + sf_kb * 4) * 512, nch * 512, &sh.sffull[slot]);
        if (b_hi)
          bulk_load(sh.sfb[slot][C::BHALVES - 1], p.sb + ((bb + 1) * c4 + sf_kb * 4) * 512, nch * 512,
                    &sh.sffull[slot]);
        sf_filled |= 1u << slot;
        sf_last = (sf_last & ~(1u << slot)) | (sf_phase << slot);
        if (++slot == SF_SLOTS) {
          slot = 0;
          sf_phase ^= 1;
        }
        if (++sf_kb == p.nkb) {
          sf_kb = 0;
          sf_tile += gridDim.x;
        }
      };
      load_scales();  // step 0
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
        for (int kb = 0; kb < p.nkb; ++kb) {
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, abort_flag, kFaultTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sh.a[stage], &tmA, &sh.full[stage], kb * BKB, tm * BM);
          tma_load_2d(sh.b[stage], &tmB, &sh.full[stage], kb * BKB, tn * BN);
          filled |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          load_scales();  // the next step's
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s)
          if (filled & (1u << s)) blockgemm::drain_wait(&sh.full[s], (last_phase >> s) & 1);
        for (int s = 0; s < SF_SLOTS; ++s)
          if (sf_filled & (1u << s)) blockgemm::drain_wait(&sh.sffull[s], (sf_last >> s) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_block_scaled(1, 1, BM, BN);  // e2m1 x e2m1, ue4m3 scales, f32 accumulate
      int stage = 0, slot = 0;
      uint32_t phase = 0, sf_phase = 0, acc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&sh.tempty, (acc & 1) ^ 1, abort_flag, kFaultTimeoutMma)) break;
        tc_fence_after();
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int nch = min(4, p.nchunk - kb * 4);
          // the step's scales are in TMEM (the scale issuers' commits) and its operands have landed
          if (!mbar_wait(&sh.sfready[slot], sf_phase, abort_flag, kFaultTimeoutMma) ||
              !mbar_wait(&sh.full[stage], phase, abort_flag, kFaultTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfcol = tmem + SF_COL0 + slot * SF_COLS_PER_STAGE;
          const uint64_t ad = desc_sw128(smem_u32(sh.a[stage]));
          const uint64_t bd = desc_sw128(smem_u32(sh.b[stage]));
          for (int c = 0; c < nch; ++c)
            mma_mxf4nvf4(tmem, ad + 2 * c, bd + 2 * c, idesc, sfcol + c * 4, sfcol + SFA_COLS + c * (BN / 32),
                         (kb | c) != 0);
          mma_commit(&sh.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (++slot == SF_SLOTS) {
            slot = 0;
            sf_phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&sh.tfull);
        ++acc;
      }
      mma_commit(&sh.mdrain);
      blockgemm::drain_wait(&sh.mdrain, 0);
    }
  } else if (warp < EPI_WARP0) {
    // scale issuers: step g's scale tiles go to its slot's TMEM columns once they have landed. The columns' previous
    // readers, the MMAs of step g - SF_SLOTS, have finished by then: the producer loaded these scales after its wait
    // on `empty` for step g - 1, which those MMAs (step g - 1 - STAGES) had committed.
    if (lane == 0) {
      const bool first = warp == 2;
      int slot = 0;
      uint32_t sf_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int tn = tile % p.tiles_n;
        const bool b_hi = C::BHALVES == 2 && (int64_t)tn * 2 + 1 < p.nblk_b;
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int nch = min(4, p.nchunk - kb * 4);
          if (!mbar_wait(&sh.sffull[slot], sf_phase, abort_flag, kFaultTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfcol = tmem + SF_COL0 + slot * SF_COLS_PER_STAGE;
          // warp 2: A's scales, and with BN = 256 those of B's first 128 rows; warp 3: the rest of B's
          if (first) {
            for (int c = 0; c < nch; ++c) {
              tmem_cp_32x128b_x4(sfcol + c * 4, desc_plain16(smem_u32(sh.sfa[slot] + c * 512)));
              if (BN == 256)
                tmem_cp_32x128b_x4(sfcol + SFA_COLS + c * 8, desc_plain16(smem_u32(sh.sfb[slot][0] + c * 512)));
            }
          } else if (BN == 128) {
            for (int c = 0; c < nch; ++c)
              tmem_cp_32x128b_x4(sfcol + SFA_COLS + c * 4, desc_plain16(smem_u32(sh.sfb[slot][0] + c * 512)));
          } else if (b_hi) {  // else the columns stay stale: they scale only output columns >= N
            for (int c = 0; c < nch; ++c)
              tmem_cp_32x128b_x4(sfcol + SFA_COLS + c * 8 + 4,
                                 desc_plain16(smem_u32(sh.sfb[slot][C::BHALVES - 1] + c * 512)));
          }
          mma_commit(&sh.sfready[slot]);
          if (++slot == SF_SLOTS) {
            slot = 0;
            sf_phase ^= 1;
          }
        }
      }
      mma_commit(&sh.mdrain);
      blockgemm::drain_wait(&sh.mdrain, 0);
    }
  } else {
    using OutT = typename blockgemm::Store<OUT>::T;
    const int ew = warp - EPI_WARP0;
    const int part = ew >> 2;   // which EPI_COLS columns of the tile
    const int quad = warp & 3;  // the TMEM lane quadrant this warp may read
    const float alpha = __ldg(p.alpha);
    uint32_t acc_cnt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int tm = tile / p.tiles_n, tn = tile - tm * p.tiles_n;
      if (!blockgemm::warp_wait(&sh.tfull, acc_cnt & 1, abort_flag, kFaultTimeoutEpilogue)) break;
      tc_fence_after();
      constexpr int EC = C::EPI_COLS;
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + part * EC;
      uint32_t r0[32], r1[32];
      tmem_ld32_issue(taddr, r0);
      if (EC == 64) tmem_ld32_issue(taddr + 32, r1);
      tmem_ld_wait32(r0);
      if (EC == 64) tmem_ld_wait32(r1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty);
      ++acc_cnt;
      // cast this lane's row, then trade chunks across the warp so that each store writes 4 rows x 128 bytes
      // (a store of one 16-byte chunk from each of 32 rows kept the SM's write path busy for most of a tile)
      constexpr int PER = blockgemm::Store<OUT>::PER;  // outputs per 16-byte chunk
      constexpr int CH = EC / PER < 8 ? EC / PER : 8;  // 16-byte chunks of a row a transpose moves (4 or 8)
      constexpr int LCH = CH == 8 ? 3 : 2;
      const OutT* bias = reinterpret_cast<const OutT*>(p.bias);
#pragma unroll
      for (int blk = 0; blk < EC / (CH * PER); ++blk) {
        const int nb = tn * BN + part * EC + blk * CH * PER;  // first column of the CH chunks
        uint4 c[CH];
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          float v[PER];
#pragma unroll
          for (int e = 0; e < PER; ++e) {
            const int col = blk * CH * PER + j * PER + e;
            v[e] = __fmul_rn(__uint_as_float(col < 32 ? r0[col] : r1[col - 32]), alpha);
          }
          // N % 16 == 0: a chunk is whole or absent
          c[j] = blockgemm::Store<OUT>::pack(v, bias && nb + j * PER < p.N ? bias + nb + j * PER : nullptr);
        }
        blockgemm::rows_to_segments<CH>(c, lane);
        const int col = nb + (lane & (CH - 1)) * PER;
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int row = tm * BM + quad * 32 + (32 / CH) * i + (lane >> LCH);
          if (row < p.M && col < p.N)
            *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.y) + (int64_t)row * p.N + col) = c[i];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace fp4gemm
}  // namespace b200
