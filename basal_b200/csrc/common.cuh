// Shared device helpers of libbasal200: status codes, the device fault word, bounded mbarrier waits, TMA loads and
// the tcgen05 (5th-generation tensor core) instructions of sm_100a as inline PTX.
#pragma once
#include <cuda_runtime.h>
#include <cuda.h>
#include <cstdint>

#include "../../include/basal200.h"

namespace b200 {

// Device-side fault bits, OR-ed into g_fault by a kernel that gave up (never a trap): the host reads and clears them
// with basal200_device_faults().
enum FaultBits : unsigned {
  kFaultTimeoutProducer = BASAL200_FAULT_TIMEOUT_PRODUCER,
  kFaultTimeoutMma = BASAL200_FAULT_TIMEOUT_MMA,
  kFaultTimeoutEpilogue = BASAL200_FAULT_TIMEOUT_EPILOGUE,
  kFaultTimeoutDrain = BASAL200_FAULT_TIMEOUT_DRAIN,
  kFaultBadId = BASAL200_FAULT_BAD_ID,
  kFaultTimeoutPeer = BASAL200_FAULT_TIMEOUT_PEER,
};

// The library is one translation unit (csrc/basal200.cu includes every kernel header), so the word is defined here.
__device__ unsigned g_fault = 0;

// A wait on an mbarrier gives up after this long (a correct pipeline waits microseconds): the kernel records a
// fault bit, tells its other roles to stop, drains what it issued and returns.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------------------------
// programmatic dependent launch: the library's kernels (but the weight quantisers) are launched so that they may
// start while the kernel before them in the stream finishes, once that kernel allows it
// ---------------------------------------------------------------------------------------------------------------
// Waits until the kernels this one may have started ahead of have completed and their writes are visible. Every
// kernel launched that way calls it before reading what an earlier kernel may have written and before its first
// store; without a kernel ahead it returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next kernel of the stream start launching (it still waits for this one in its pdl_wait). The weight
// quantisers never call it, so what follows them (a GEMM that loads weights before its pdl_wait) starts only after
// the weights are written.
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete. Returns false when the CTA's abort flag is set (another role gave
// up) or when this wait passes kWaitLimitNs (then it sets the abort flag and the fault bit itself).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned fault) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      atomicOr(&g_fault, fault);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) loads and stores, and the plain bulk copy
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Tiled shared -> global store of one box (bulk-group completion), and its group bookkeeping.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the smem sources of every committed store group have been read (the buffer may be rewritten).
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until every committed store group has completed (its writes are visible).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// A named barrier that also ANDs a flag over its threads: every thread leaves with the same answer (so a group whose
// members saw different outcomes of a bounded wait still takes the same branch afterwards).
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\tbarrier.red.and.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(threads), "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// Contiguous global -> shared copy; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads
// ---------------------------------------------------------------------------------------------------------------
// Allocation and release are warp-wide (.sync.aligned): call from one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA with 128-byte swizzle: rows of 128 bytes,
// 8-row groups 1024 bytes apart (stride byte offset), descriptor version 1 (sm_100), layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Descriptor of a no-swizzle K-major tile of 16-byte rows, 8-row core matrices 128 bytes apart: the source of
// tcgen05.cp's 32x128b shape (32 rows x 16 bytes, contiguous).
__device__ __forceinline__ uint64_t desc_plain16(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// Instruction descriptors (kind::f16 / f8f6f4 / i8 layout): D format bits 4-5, A format 7-9, B format 10-12, both
// operands K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_dense(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, int M, int N) {
  return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Block-scaled kinds: A/B format bits 7-9 / 10-12, scale format bit 23 (0 = ue4m3), scale-factor ids 0.
__host__ __device__ constexpr uint32_t idesc_block_scaled(uint32_t afmt, uint32_t bfmt, int M, int N) {
  return (afmt << 7) | (bfmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_mxf4nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%4], [%5], p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Copies 32 rows x 16 bytes of shared memory into 4 TMEM columns of every lane quadrant (lane l gets row l % 32).
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 columns of 32 bits: thread i of the warp gets lane (quadrant base + i), columns taddr .. taddr+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 columns of 32 bits.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32 bits, issued without waiting: the registers hold the columns only after
// tmem_ld_wait32 on the same array, which names them as operands so that no use of them can move above the wait.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait32(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// packed fp32 pairs (sm_100 f32x2 arithmetic) and register reallocation between warpgroups
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ uint64_t pack_u2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

__device__ __forceinline__ float2 unpack_f2(uint64_t v) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
  return f;
}

// acc = {lo, hi} * s2 + acc, both lanes rounded once (fma.rn.f32x2).
__device__ __forceinline__ void ffma2(uint64_t& acc, uint32_t lo, uint32_t hi, uint64_t s2) {
  asm("{\n\t.reg .b64 t;\n\tmov.b64 t, {%1, %2};\n\tfma.rn.f32x2 %0, t, %3, %0;\n\t}"
      : "+l"(acc)
      : "r"(lo), "r"(hi), "l"(s2));
}

// 64 consecutive TMEM columns of this warp's 32 lanes (two 32x32b.x32 loads, then the wait), returned as 32 packed
// fp32 pairs (columns 2j, 2j+1) ready for f32x2 arithmetic. The loads, the wait and the packing are one asm block so
// that the pairs need no register moves. INT8: the s32 partials (below 2^21 in magnitude for a 128-deep slice) are
// converted to fp32 exactly first. (Measured on B200: cvt beats the integer-add / packed-subtract conversion.)
template <bool INT8>
__device__ __forceinline__ void tmem_ld64_pairs(uint32_t taddr, uint64_t (&d)[32]) {
  if (INT8) {
    asm volatile("{\n\t.reg .b32 a0,a1,a2,a3,a4,a5,a6,a7,a8,a9,a10,a11,a12,a13,a14,a15,a16,a17,a18,a19,a20,a21,a22,a23,a24,a25,a26,a27,a28,a29,a30,a31,a32,a33,a34,a35,a36,a37,a38,a39,a40,a41,a42,a43,a44,a45,a46,a47,a48,a49,a50,a51,a52,a53,a54,a55,a56,a57,a58,a59,a60,a61,a62,a63;\n\ttcgen05.ld.sync.aligned.32x32b.x32.b32 {a0,a1,a2,a3,a4,a5,a6,a7,a8,a9,a10,a11,a12,a13,a14,a15,a16,a17,a18,a19,a20,a21,a22,a23,a24,a25,a26,a27,a28,a29,a30,a31}, [%32];\n\ttcgen05.ld.sync.aligned.32x32b.x32.b32 {a32,a33,a34,a35,a36,a37,a38,a39,a40,a41,a42,a43,a44,a45,a46,a47,a48,a49,a50,a51,a52,a53,a54,a55,a56,a57,a58,a59,a60,a61,a62,a63}, [%33];\n\ttcgen05.wait::ld.sync.aligned;\n\tcvt.rn.f32.s32 a0, a0;\n\tcvt.rn.f32.s32 a1, a1;\n\tcvt.rn.f32.s32 a2, a2;\n\tcvt.rn.f32.s32 a3, a3;\n\tcvt.rn.f32.s32 a4, a4;\n\tcvt.rn.f32.s32 a5, a5;\n\tcvt.rn.f32.s32 a6, a6;\n\tcvt.rn.f32.s32 a7, a7;\n\tcvt.rn.f32.s32 a8, a8;\n\tcvt.rn.f32.s32 a9, a9;\n\tcvt.rn.f32.s32 a10, a10;\n\tcvt.rn.f32.s32 a11, a11;\n\tcvt.rn.f32.s32 a12, a12;\n\tcvt.rn.f32.s32 a13, a13;\n\tcvt.rn.f32.s32 a14, a14;\n\tcvt.rn.f32.s32 a15, a15;\n\tcvt.rn.f32.s32 a16, a16;\n\tcvt.rn.f32.s32 a17, a17;\n\tcvt.rn.f32.s32 a18, a18;\n\tcvt.rn.f32.s32 a19, a19;\n\tcvt.rn.f32.s32 a20, a20;\n\tcvt.rn.f32.s32 a21, a21;\n\tcvt.rn.f32.s32 a22, a22;\n\tcvt.rn.f32.s32 a23, a23;\n\tcvt.rn.f32.s32 a24, a24;\n\tcvt.rn.f32.s32 a25, a25;\n\tcvt.rn.f32.s32 a26, a26;\n\tcvt.rn.f32.s32 a27, a27;\n\tcvt.rn.f32.s32 a28, a28;\n\tcvt.rn.f32.s32 a29, a29;\n\tcvt.rn.f32.s32 a30, a30;\n\tcvt.rn.f32.s32 a31, a31;\n\tcvt.rn.f32.s32 a32, a32;\n\tcvt.rn.f32.s32 a33, a33;\n\tcvt.rn.f32.s32 a34, a34;\n\tcvt.rn.f32.s32 a35, a35;\n\tcvt.rn.f32.s32 a36, a36;\n\tcvt.rn.f32.s32 a37, a37;\n\tcvt.rn.f32.s32 a38, a38;\n\tcvt.rn.f32.s32 a39, a39;\n\tcvt.rn.f32.s32 a40, a40;\n\tcvt.rn.f32.s32 a41, a41;\n\tcvt.rn.f32.s32 a42, a42;\n\tcvt.rn.f32.s32 a43, a43;\n\tcvt.rn.f32.s32 a44, a44;\n\tcvt.rn.f32.s32 a45, a45;\n\tcvt.rn.f32.s32 a46, a46;\n\tcvt.rn.f32.s32 a47, a47;\n\tcvt.rn.f32.s32 a48, a48;\n\tcvt.rn.f32.s32 a49, a49;\n\tcvt.rn.f32.s32 a50, a50;\n\tcvt.rn.f32.s32 a51, a51;\n\tcvt.rn.f32.s32 a52, a52;\n\tcvt.rn.f32.s32 a53, a53;\n\tcvt.rn.f32.s32 a54, a54;\n\tcvt.rn.f32.s32 a55, a55;\n\tcvt.rn.f32.s32 a56, a56;\n\tcvt.rn.f32.s32 a57, a57;\n\tcvt.rn.f32.s32 a58, a58;\n\tcvt.rn.f32.s32 a59, a59;\n\tcvt.rn.f32.s32 a60, a60;\n\tcvt.rn.f32.s32 a61, a61;\n\tcvt.rn.f32.s32 a62, a62;\n\tcvt.rn.f32.s32 a63, a63;\n\tmov.b64 %0, {a0, a1};\n\tmov.b64 %1, {a2, a3};\n\tmov.b64 %2, {a4, a5};\n\tmov.b64 %3, {a6, a7};\n\tmov.b64 %4, {a8, a9};\n\tmov.b64 %5, {a10, a11};\n\tmov.b64 %6, {a12, a13};\n\tmov.b64 %7, {a14, a15};\n\tmov.b64 %8, {a16, a17};\n\tmov.b64 %9, {a18, a19};\n\tmov.b64 %10, {a20, a21};\n\tmov.b64 %11, {a22, a23};\n\tmov.b64 %12, {a24, a25};\n\tmov.b64 %13, {a26, a27};\n\tmov.b64 %14, {a28, a29};\n\tmov.b64 %15, {a30, a31};\n\tmov.b64 %16, {a32, a33};\n\tmov.b64 %17, {a34, a35};\n\tmov.b64 %18, {a36, a37};\n\tmov.b64 %19, {a38, a39};\n\tmov.b64 %20, {a40, a41};\n\tmov.b64 %21, {a42, a43};\n\tmov.b64 %22, {a44, a45};\n\tmov.b64 %23, {a46, a47};\n\tmov.b64 %24, {a48, a49};\n\tmov.b64 %25, {a50, a51};\n\tmov.b64 %26, {a52, a53};\n\tmov.b64 %27, {a54, a55};\n\tmov.b64 %28, {a56, a57};\n\tmov.b64 %29, {a58, a59};\n\tmov.b64 %30, {a60, a61};\n\tmov.b64 %31, {a62, a63};\n\t}"
                 : "=l"(d[0]), "=l"(d[1]), "=l"(d[2]), "=l"(d[3]), "=l"(d[4]), "=l"(d[5]), "=l"(d[6]), "=l"(d[7]), "=l"(d[8]), "=l"(d[9]), "=l"(d[10]), "=l"(d[11]), "=l"(d[12]), "=l"(d[13]), "=l"(d[14]), "=l"(d[15]), "=l"(d[16]), "=l"(d[17]), "=l"(d[18]), "=l"(d[19]), "=l"(d[20]), "=l"(d[21]), "=l"(d[22]), "=l"(d[23]), "=l"(d[24]), "=l"(d[25]), "=l"(d[26]), "=l"(d[27]), "=l"(d[28]), "=l"(d[29]), "=l"(d[30]), "=l"(d[31])
                 : "r"(taddr), "r"(taddr + 32)
                 : "memory");
  } else {
    asm volatile("{\n\t.reg .b32 a0,a1,a2,a3,a4,a5,a6,a7,a8,a9,a10,a11,a12,a13,a14,a15,a16,a17,a18,a19,a20,a21,a22,a23,a24,a25,a26,a27,a28,a29,a30,a31,a32,a33,a34,a35,a36,a37,a38,a39,a40,a41,a42,a43,a44,a45,a46,a47,a48,a49,a50,a51,a52,a53,a54,a55,a56,a57,a58,a59,a60,a61,a62,a63;\n\ttcgen05.ld.sync.aligned.32x32b.x32.b32 {a0,a1,a2,a3,a4,a5,a6,a7,a8,a9,a10,a11,a12,a13,a14,a15,a16,a17,a18,a19,a20,a21,a22,a23,a24,a25,a26,a27,a28,a29,a30,a31}, [%32];\n\ttcgen05.ld.sync.aligned.32x32b.x32.b32 {a32,a33,a34,a35,a36,a37,a38,a39,a40,a41,a42,a43,a44,a45,a46,a47,a48,a49,a50,a51,a52,a53,a54,a55,a56,a57,a58,a59,a60,a61,a62,a63}, [%33];\n\ttcgen05.wait::ld.sync.aligned;\n\tmov.b64 %0, {a0, a1};\n\tmov.b64 %1, {a2, a3};\n\tmov.b64 %2, {a4, a5};\n\tmov.b64 %3, {a6, a7};\n\tmov.b64 %4, {a8, a9};\n\tmov.b64 %5, {a10, a11};\n\tmov.b64 %6, {a12, a13};\n\tmov.b64 %7, {a14, a15};\n\tmov.b64 %8, {a16, a17};\n\tmov.b64 %9, {a18, a19};\n\tmov.b64 %10, {a20, a21};\n\tmov.b64 %11, {a22, a23};\n\tmov.b64 %12, {a24, a25};\n\tmov.b64 %13, {a26, a27};\n\tmov.b64 %14, {a28, a29};\n\tmov.b64 %15, {a30, a31};\n\tmov.b64 %16, {a32, a33};\n\tmov.b64 %17, {a34, a35};\n\tmov.b64 %18, {a36, a37};\n\tmov.b64 %19, {a38, a39};\n\tmov.b64 %20, {a40, a41};\n\tmov.b64 %21, {a42, a43};\n\tmov.b64 %22, {a44, a45};\n\tmov.b64 %23, {a46, a47};\n\tmov.b64 %24, {a48, a49};\n\tmov.b64 %25, {a50, a51};\n\tmov.b64 %26, {a52, a53};\n\tmov.b64 %27, {a54, a55};\n\tmov.b64 %28, {a56, a57};\n\tmov.b64 %29, {a58, a59};\n\tmov.b64 %30, {a60, a61};\n\tmov.b64 %31, {a62, a63};\n\t}"
                 : "=l"(d[0]), "=l"(d[1]), "=l"(d[2]), "=l"(d[3]), "=l"(d[4]), "=l"(d[5]), "=l"(d[6]), "=l"(d[7]), "=l"(d[8]), "=l"(d[9]), "=l"(d[10]), "=l"(d[11]), "=l"(d[12]), "=l"(d[13]), "=l"(d[14]), "=l"(d[15]), "=l"(d[16]), "=l"(d[17]), "=l"(d[18]), "=l"(d[19]), "=l"(d[20]), "=l"(d[21]), "=l"(d[22]), "=l"(d[23]), "=l"(d[24]), "=l"(d[25]), "=l"(d[26]), "=l"(d[27]), "=l"(d[28]), "=l"(d[29]), "=l"(d[30]), "=l"(d[31])
                 : "r"(taddr), "r"(taddr + 32)
                 : "memory");
  }
}

// acc = x * s2 + acc on packed fp32 pairs (fma.rn.f32x2, each lane rounded once).
__device__ __forceinline__ void ffma2p(uint64_t& acc, uint64_t x, uint64_t s2) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(x), "l"(s2));
}

template <uint32_t N>
__device__ __forceinline__ void regs_release() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

template <uint32_t N>
__device__ __forceinline__ void regs_claim() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ int warp_id() { return __shfl_sync(0xffffffffu, threadIdx.x / 32, 0); }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace b200
