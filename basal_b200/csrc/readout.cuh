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

// code_logits on the tensor cores, for h and head of one 16-bit type (bf16 or fp16) whose rows start on 16-byte
// boundaries, D % 8 == 0. A tile is 128 prompts x BN codes (BN = 16 or 32); its features are cut into 8 slices of
// tc_slice(D) features (whole 64-feature swizzle rows; the last slices shorter or empty), and a cluster of 8 CTAs
// takes one tile, CTA s the slice s:
//   1. its 128 prompt rows and BN code rows (gathered by id) of the slice are copied into shared memory with 16-byte
//      cp.async in the 128-byte-swizzled K-major layout tcgen05 reads (zeros past D, past R and for a bad id), up to
//      tkr<BN>() features a round;
//   2. one thread chains tcgen05.mma kind::f16 over the slice's 16-feature steps in increasing feature order into
//      one fp32 TMEM accumulator (128 lanes x BN columns): bf16 x bf16 products are exact in fp32;
//   3. warps 0-3 read the accumulator (a row a thread); each thread pushes its row's BN sums into the slot of its
//      slice in the CTA that owns the row (CTA k owns rows 16 k .. 16 k + 15 of the tile), with st.async stores that
//      count down the owner's mbarrier;
//   4. once the 8 slots of its rows have landed, CTA k adds them in slice order 0, 1, .., 7 (fp32, round to
//      nearest), adds the bias, applies the soft cap and stores z.
// Every z[r, u] is therefore one fixed function of h[r, :], the code's row and D: the slices, the steps of each
// chain and the order of the slices depend on D alone, never on R, U, BN or where the prompt and the code sit in
// their tiles (the contract of CodeReadout.probs_each, readout.py:86-104). Eight slices also keep each chain short,
// and with it the tensor core's fp32 accumulation error.
constexpr int TM = 128;       // prompts a tile (the MMA's M)
constexpr int TSPLIT = 8;     // feature slices a tile = CTAs a cluster
constexpr int TKR = 320;      // most features a CTA stages in one round (5 rows of the 128-byte swizzle)
// features a round for BN codes: 256 with 32 codes keeps two CTAs on an SM (a cluster needs 8 CTAs in one GPC)
template <int BN>
constexpr int tkr() { return BN == 32 ? 256 : TKR; }
constexpr int TTHREADS = 256; // 8 warps issue the copies; warps 0-3 read the accumulators
constexpr int TROWS = TM / TSPLIT;  // rows of the tile a CTA owns in step 4

__host__ __device__ constexpr int64_t tc_slice(int64_t D) { return (D + TSPLIT * 64 - 1) / (TSPLIT * 64) * 64; }

template <int BN>
struct TcSmem {
  uint8_t a[tkr<BN>() / 64][TM * 128];  // 1024-byte aligned (the struct is placed on a 1024-byte boundary)
  uint8_t b[tkr<BN>() / 64][BN * 128];
  float recv[TSPLIT][TROWS][BN];   // slot s: the sums of slice s for the rows this CTA owns (pushed by CTA s)
  int recv_ok[TSPLIT];             // slot s: CTA s completed its MMAs
  int64_t id[BN];                  // each code's row of the head (-1: past U or a bad id)
  uint64_t done;                   // the MMAs of a round completed
  uint64_t got;                    // every slot of recv and recv_ok landed
  uint32_t tmem;
  int abort;
  int abort_got;
};
template <int BN>
constexpr size_t tc_smem_bytes() { return sizeof(TcSmem<BN>) + 1024; }
template <int BN>
constexpr uint32_t tc_recv_bytes() { return TSPLIT * TROWS * BN * 4 + TSPLIT * 4; }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Stores into another CTA's shared memory (a cluster address) that complete_tx its mbarrier by their bytes.
__device__ __forceinline__ void st_async_f4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
               ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void st_async_s32(uint32_t addr, int v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.s32 [%0], %1, [%2];" ::"r"(addr), "r"(v),
               "r"(bar)
               : "memory");
}

// The softmax of one prompt's codes, lane l holding codes l, l + 32, .. (-inf: padding or past Kmax): max, exp, sum
// and division in this order, so any NI at least the prompt's width gives the same bits (a -inf code adds nothing).
template <int NI>
__device__ __forceinline__ void softmax_lanes(float (&v)[NI]) {
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NI; ++i) m = fmaxf(m, v[i]);
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
  for (int i = 0; i < NI; ++i) v[i] = __fdiv_rn(v[i], s);
}

template <typename T, typename TB, int BN>
__global__ void __launch_bounds__(TTHREADS) code_logits_tc_kernel(
    const T* __restrict__ h, int64_t R, int64_t D, int64_t ldh, const T* __restrict__ head, int64_t V, int64_t ldw,
    const int64_t* __restrict__ ids, int64_t U, const TB* __restrict__ bias, float softcap, float* __restrict__ z) {
  static_assert(sizeof(T) == 2 && (BN == 16 || BN == 32), "16-bit rows, 16 or 32 codes a tile");
  constexpr uint32_t IDESC = idesc_dense(1, std::is_same<T, __nv_bfloat16>::value ? 1 : 0,
                                         std::is_same<T, __nv_bfloat16>::value ? 1 : 0, TM, BN);
  constexpr uint32_t NCOLS = 32;  // the accumulator's BN <= 32 columns (the smallest allocation)
  extern __shared__ uint8_t smem_raw[];
  TcSmem<BN>& sh = *reinterpret_cast<TcSmem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t m0 = (int64_t)blockIdx.x * TM, n0 = (int64_t)blockIdx.y * BN;
  const int slice = (int)blockIdx.z;  // the CTA's rank in its cluster (cluster dims 1 x 1 x 8)
  const int64_t KS = tc_slice(D);
  const int64_t f_begin = slice * KS;
  const int64_t f_end = f_begin + KS < D ? f_begin + KS : D;  // <= f_begin: an empty slice
  if (tid == 0) {
    mbar_init(&sh.done, 1);
    mbar_init(&sh.got, 1);
    sh.abort = 0;
    sh.abort_got = 0;
    mbar_arrive_expect_tx(&sh.got, tc_recv_bytes<BN>());  // the 8 CTAs' pushes complete its first phase
    fence_barrier_init();
  }
  __syncthreads();
  cluster_arrive_relaxed();  // the barriers' init is released by its fence: the others push after their wait
  pdl_launch();
  pdl_wait();
  int64_t id = tid < BN && n0 + tid < U ? __ldg(ids + n0 + tid) : -1;  // in flight while the prompt rows are asked for
  // the code row this thread copies (thread t: row t / 8), its id loaded by the thread itself, so that its copies go
  // out as soon as the id arrives
  const int brow = tid >> 3;
  int64_t bid = brow < BN && n0 + brow < U ? __ldg(ids + n0 + brow) : -1;
  // 1. copies: 8 consecutive threads take the 8 16-byte chunks of one row's 128-byte swizzle row
  constexpr int KR = tkr<BN>();
  const int cc = tid & 7;
  auto copy_prompts = [&](int64_t g0, int64_t g1, int natoms) {
    for (int atom = 0; atom < natoms; ++atom) {
#pragma unroll
      for (int r = tid >> 3; r < TM; r += TTHREADS / 8) {
        const int64_t f = g0 + atom * 64 + cc * 8;
        const bool in = m0 + r < R && f < g1;
        cp_async16(smem_u32(sh.a[atom]) + blockgemm::sw128(r, cc), in ? h + (m0 + r) * ldh + f : h, in ? 16u : 0u);
      }
    }
  };
  auto round_end = [&](int64_t g0) { return g0 + KR < f_end ? g0 + KR : f_end; };
  auto round_atoms = [&](int64_t g0) { return (int)((round_end(g0) - g0 + 63) / 64); };
  if (f_begin < f_end) copy_prompts(f_begin, round_end(f_begin), round_atoms(f_begin));
  if (bid < 0 || bid >= V) bid = -1;
  auto copy_codes = [&](int64_t g0, int64_t g1, int natoms) {
    if (brow < BN) {
      for (int atom = 0; atom < natoms; ++atom) {
        const int64_t f = g0 + atom * 64 + cc * 8;
        const bool in = bid >= 0 && f < g1;
        cp_async16(smem_u32(sh.b[atom]) + blockgemm::sw128(brow, cc), in ? head + bid * ldw + f : head, in ? 16u : 0u);
      }
    }
  };
  if (f_begin < f_end) copy_codes(f_begin, round_end(f_begin), round_atoms(f_begin));
  if (warp == 0) tmem_alloc(&sh.tmem, NCOLS);
  if (tid < BN) {
    if (n0 + tid < U && (id < 0 || id >= V)) {
      if (blockIdx.x == 0 && slice == 0) atomicOr(&g_fault, kFaultBadId);
      id = -1;
    }
    sh.id[tid] = id;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  bool ok = true;
  int steps = 0;  // MMA steps issued so far
  uint32_t phase = 0;
  for (int64_t g0 = f_begin; g0 < f_end && ok; g0 += KR) {
    const int64_t g1 = round_end(g0);
    const int natoms = round_atoms(g0);
    if (g0 != f_begin) {
      copy_prompts(g0, g1, natoms);
      copy_codes(g0, g1, natoms);
    }
    cp_async_wait_all();
    fence_proxy_async();  // the copies (generic proxy) before the tensor core's reads (async proxy)
    __syncthreads();
    // 2. the round's MMA steps, in feature order
    const int nsteps = (int)((g1 - g0 + 15) / 16);
    if (tid == 0) {
      tc_fence_after();
      // step i reads 32 bytes at (i & 3) * 32 of swizzle row i >> 2: descriptor address fields count 16 bytes
      const uint64_t a0 = desc_sw128(smem_u32(sh.a[0])), b0 = desc_sw128(smem_u32(sh.b[0]));
#pragma unroll 4
      for (int i = 0; i < nsteps; ++i) {
        const uint64_t k = (uint64_t)((i & 3) * 2);
        mma_f16(tmem, a0 + (uint64_t)(i >> 2) * (TM * 128 / 16) + k, b0 + (uint64_t)(i >> 2) * (BN * 128 / 16) + k,
                IDESC, steps + i > 0 ? 1u : 0u);
      }
      mma_commit(&sh.done);
    }
    steps += nsteps;
    ok = mbar_wait(&sh.done, phase, &sh.abort, kFaultTimeoutMma);
    if (!__syncthreads_and(ok)) {  // the MMAs never completed: wait (bounded) for them, keep the shared memory
      if (tid == 0) blockgemm::drain_wait(&sh.done, phase);
      __syncthreads();
      ok = false;
    }
    phase ^= 1;
  }
  // 3. warps 0-3: the row's sums (zero for an empty slice or after a failed wait), pushed to the row's owner
  float acc[BN];
  if (warp < 4 && ok && steps > 0) {
    tc_fence_after();
    uint32_t v[BN];
    if constexpr (BN == 32) {
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
    } else {
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), v);
    }
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < BN; ++j) acc[j] = __uint_as_float(v[j]);
  } else {
#pragma unroll
    for (int j = 0; j < BN; ++j) acc[j] = 0.0f;
  }
  cluster_wait();  // every CTA of the cluster has initialised its barriers
  if (warp < 4) {
    const uint32_t owner = (uint32_t)(tid / TROWS);
    const uint32_t dst = cluster_map(smem_u32(&sh.recv[slice][tid % TROWS][0]), owner);
    const uint32_t bar = cluster_map(smem_u32(&sh.got), owner);
#pragma unroll
    for (int j = 0; j < BN; j += 4) st_async_f4(dst + j * 4, acc[j], acc[j + 1], acc[j + 2], acc[j + 3], bar);
  }
  if (tid < TSPLIT)
    st_async_s32(cluster_map(smem_u32(&sh.recv_ok[slice]), (uint32_t)tid), ok ? 1 : 0,
                 cluster_map(smem_u32(&sh.got), (uint32_t)tid));
  // 4. rows 16 s .. 16 s + 15 of the tile: the 8 slots in slice order, the bias and the soft cap, z
  const bool got = mbar_wait(&sh.got, 0, &sh.abort_got, kFaultTimeoutEpilogue);
  constexpr int Q = BN / 4;  // float4 columns a row
  if (got && tid < TROWS * Q) {
    const int rl = tid / Q, c0 = (tid % Q) * 4;
    float4 s4 = *reinterpret_cast<const float4*>(&sh.recv[0][rl][c0]);
    int all_ok = sh.recv_ok[0];
#pragma unroll
    for (int k = 1; k < TSPLIT; ++k) {
      const float4 p4 = *reinterpret_cast<const float4*>(&sh.recv[k][rl][c0]);
      all_ok &= sh.recv_ok[k];
      s4.x = __fadd_rn(s4.x, p4.x);
      s4.y = __fadd_rn(s4.y, p4.y);
      s4.z = __fadd_rn(s4.z, p4.z);
      s4.w = __fadd_rn(s4.w, p4.w);
    }
    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
    const int64_t r = m0 + slice * TROWS + rl;
    if (all_ok && r < R) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t u = n0 + c0 + e;
        if (u < U) {
          float v = sv[e];
          const int64_t cid = sh.id[c0 + e];
          if (cid < 0) {
            v = __int_as_float(0x7fc00000);
          } else if (bias) {
            v = __fadd_rn(v, load1(bias + cid));
          }
          if (softcap > 0.0f) v = __fmul_rn(tanhf(__fdiv_rn(v, softcap)), softcap);
          z[r * U + u] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, NCOLS);
  }
}

// One warp per prompt row, NI <= 32 codes a lane (Kmax <= 32 NI): every index, padding flag and logit is loaded
// before any arithmetic, then max, exp, sum and division in the same order for every NI. The indices and padding flags
// are inputs of the readout, never results of the kernel ahead (code_logits), so they are read before the wait for
// it: their latency overlaps that kernel. When a row of z has at most ZROW logits the warp then reads the whole row
// into shared memory (coalesced) and gathers from there instead of from scattered addresses.
constexpr int ZROW = 1024;

template <int NI>
__global__ void __launch_bounds__(256) code_probs_kernel(const float* __restrict__ z, int64_t R, int64_t U,
                                                         const int64_t* __restrict__ idx,
                                                         const uint8_t* __restrict__ pad, int64_t Kmax,
                                                         float* __restrict__ p) {
  __shared__ float zs[8][ZROW];
  pdl_launch();
  const int64_t r = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (r >= R) return;
  const bool stage = U <= ZROW;
  int64_t c[NI];
  bool use[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int64_t j = lane + 32 * i;
    const bool in = j < Kmax;
    c[i] = in ? __ldg(idx + r * Kmax + j) : -1;
    use[i] = in && !(pad && __ldg(pad + r * Kmax + j));
  }
  pdl_wait();
  if (stage) {
    float zr[ZROW / 32];
#pragma unroll
    for (int t = 0; t < ZROW / 32; ++t) zr[t] = lane + 32 * t < U ? z[r * U + lane + 32 * t] : 0.0f;
#pragma unroll
    for (int t = 0; t < ZROW / 32; ++t) zs[w][lane + 32 * t] = zr[t];
    __syncwarp();
  }
  float v[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i)
    v[i] = (use[i] && c[i] >= 0 && c[i] < U) ? (stage ? zs[w][c[i]] : z[r * U + c[i]]) : -INFINITY;
  softmax_lanes<NI>(v);
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int64_t j = lane + 32 * i;
    if (j < Kmax) p[r * Kmax + j] = v[i];
  }
}

}  // namespace readout
}  // namespace b200
