// libbasal200: host side of the C ABI declared in include/basal200.h, and the one translation unit that holds every
// kernel of the library (the device fault word is shared by all of them).
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "block_gemm.cuh"
#include "small_gemm.cuh"
#include "nvfp4_gemm.cuh"
#include "quant.cuh"
#include "readout.cuh"
#include "hybrid.cuh"
#include "gdn_chunk.cuh"

namespace b200 {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int checked = 0;  // 1: sm_100, -1: another architecture
  int sms = 0;
  uint64_t smem_set[2] = {0, 0};  // kernels whose dynamic shared memory limit was raised on this device
};
DeviceInfo g_dev[kMaxDevices];

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kMaxDevices) return BASAL200_ERR_LAUNCH;
  DeviceInfo& d = g_dev[*dev];
  if (!d.checked) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, *dev);
    d.checked = (major == 10 && minor == 0) ? 1 : -1;
  }
  return d.checked == 1 ? BASAL200_OK : BASAL200_ERR_ARCH;
}

// Bits of DeviceInfo::smem_set, one per kernel instantiation that needs more than the default shared memory.
enum SmemSlot {
  kSlotBlock = 0, kSlotFp4 = 8, kSlotSmall = 14, kSlotSplit = 26, kSlotSplitQ = 30, kSlotLogits = 38, kSlotGlu = 50,
  kSlotRes = 58, kSlotGdn = 62, kSlotLogitsTc = 64, kSlotGdnV = 76, kSlotGdnVO = 78
};
// kSlotFp4 .. + 5, kSlotSmall .. + 11, kSlotSplit .. + 3, kSlotSplitQ .. + 7, kSlotLogits .. + 11, kSlotGlu .. + 7,
// kSlotRes .. + 3, kSlotGdn, kSlotLogitsTc .. + 11, kSlotGdnV .. + 1, kSlotGdnVO .. + 1 (bits of a 128-bit mask)

bool smem_is_set(int dev, int slot) { return (g_dev[dev].smem_set[slot >> 6] >> (slot & 63)) & 1; }

// Raises the dynamic shared-memory limit of `kernel` once per device (bit `slot` of the device's mask).
template <typename K>
int set_smem(int dev, int slot, K kernel, size_t bytes) {
  DeviceInfo& d = g_dev[dev];
  if (smem_is_set(dev, slot)) return BASAL200_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return BASAL200_ERR_LAUNCH;
  d.smem_set[slot >> 6] |= 1ull << (slot & 63);
  return BASAL200_OK;
}

int launched() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "libbasal200: launch failed: %s\n", cudaGetErrorString(e));
    return BASAL200_ERR_LAUNCH;
  }
  return BASAL200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// A 2-D byte matrix [outer, inner] with rows `row_bytes` apart, read in boxes of [box_outer, box_inner] bytes with
// the 128-byte swizzle; out-of-range elements read as zero.
int tmap_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
            uint32_t box_inner, uint32_t box_outer) {
  EncodeTiled fn = encode_fn();
  if (!fn) return BASAL200_ERR_TMAP;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BASAL200_OK : BASAL200_ERR_TMAP;
}

// A 2-D matrix of 16-bit elements [outer, inner] read / written in boxes of [box_outer, box_inner] elements with the
// 128-byte swizzle (box_inner * 2 must be 128).
int tmap_u16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
             uint32_t box_outer) {
  EncodeTiled fn = encode_fn();
  if (!fn) return BASAL200_ERR_TMAP;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BASAL200_OK : BASAL200_ERR_TMAP;
}

int grid_for(int dev, int64_t work_items, int per_block) {
  const int64_t want = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)g_dev[dev].sms * 16;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

// Launches a kernel that may start while the kernel before it in the stream finishes, once that one allows it
// (programmatic stream serialization). The kernel calls pdl_wait() before reading any earlier kernel's output and
// before its first store. The weight quantisers are launched plainly and never allow an early start.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) != cudaSuccess) return launched();
  return launched();
}

// ------------------------------------------------------------------------------------------------------------
// quantisers
// ------------------------------------------------------------------------------------------------------------
// A quantiser lets the next kernel launch at its start when its grid is one resident wave (the next kernel's CTAs
// then take no SM it still needs), else after its work. `per_sm` = the quantiser's CTAs an SM holds at once.
int early_trigger(int dev, int64_t grid, int per_sm) { return grid <= (int64_t)g_dev[dev].sms * per_sm ? 1 : 0; }

// PAIRS > 0: act_quant_block_kernel with PAIRS group pairs a warp; PAIRS < 0: act_quant_wide_kernel with -PAIRS
// steps of 4 groups a warp.
template <bool INT8, int PAIRS, typename T>
int act_quant_launch_t(const void* x, int64_t groups, uint8_t* q, float* s, int grid, cudaStream_t st, int early) {
  if constexpr (PAIRS > 0)
    return launch_pdl(act_quant_block_kernel<T, INT8, PAIRS>, grid, 256, 0, st, static_cast<const T*>(x), groups, q,
                      s, early);
  else
    return launch_pdl(act_quant_wide_kernel<T, INT8, -PAIRS, 4>, grid, 256, 0, st, static_cast<const T*>(x), groups, q,
                      s, early);
}

template <bool INT8, int PAIRS>
int act_quant_launch(const void* x, int xt, int64_t groups, uint8_t* q, float* s, int grid, cudaStream_t st,
                     int early) {
  switch (xt) {
    case BASAL200_BF16:
      return act_quant_launch_t<INT8, PAIRS, __nv_bfloat16>(x, groups, q, s, grid, st, early);
    case BASAL200_F16:
      return act_quant_launch_t<INT8, PAIRS, __half>(x, groups, q, s, grid, st, early);
    case BASAL200_F32:
      return act_quant_launch_t<INT8, PAIRS, float>(x, groups, q, s, grid, st, early);
    default:
      return BASAL200_ERR_DTYPE;
  }
}

template <bool INT8>
int act_quant(const void* x, int xt, int64_t M, int64_t K, void* q, float* s, cudaStream_t st) {
  if (M < 0 || K <= 0) return BASAL200_ERR_ARG;
  if (K % 128) return BASAL200_ERR_SHAPE;
  if (M == 0) return BASAL200_OK;
  if (!x || !q || !s) return BASAL200_ERR_ARG;
  if (!aligned16(x) || !aligned16(q) || !aligned16(s)) return BASAL200_ERR_ALIGN;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t groups = M * (K / 128);
  uint8_t* qb = static_cast<uint8_t*>(q);
  // 8 warps a CTA; once every SM gets 16 CTAs of 8 groups a warp: the wide kernel (4 lanes a group, 1 step of 8
  // groups a warp)
  if (groups >= (int64_t)g_dev[dev].sms * 16 * 64) {
    const int grid = grid_for(dev, groups, 64);
    return act_quant_launch<INT8, -1>(x, xt, groups, qb, s, grid, st, early_trigger(dev, grid, 3));
  }
  const int grid = grid_for(dev, groups, 16);
  return act_quant_launch<INT8, 1>(x, xt, groups, qb, s, grid, st, early_trigger(dev, grid, 4));
}

template <bool INT8>
int weight_quant(const void* w, int wt, int64_t N, int64_t K, void* q, float* s, cudaStream_t st) {
  if (N <= 0 || K <= 0 || !w || !q || !s) return BASAL200_ERR_ARG;
  if (N % 128 || K % 128) return BASAL200_ERR_SHAPE;
  if (!aligned16(w) || !aligned16(q)) return BASAL200_ERR_ALIGN;
  if (N / 128 > 65535) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const dim3 grid((unsigned)(K / 128), (unsigned)(N / 128));
  uint8_t* qb = static_cast<uint8_t*>(q);
  switch (wt) {
    case BASAL200_BF16:
      weight_quant_block_kernel<__nv_bfloat16, INT8><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), K,
                                                                           qb, s);
      break;
    case BASAL200_F16:
      weight_quant_block_kernel<__half, INT8><<<grid, 256, 0, st>>>(static_cast<const __half*>(w), K, qb, s);
      break;
    case BASAL200_F32:
      weight_quant_block_kernel<float, INT8><<<grid, 256, 0, st>>>(static_cast<const float*>(w), K, qb, s);
      break;
    default:
      return BASAL200_ERR_DTYPE;
  }
  return launched();
}

int nvfp4_act(const void* x, int xt, const float* inv_g, int64_t M, int64_t K, uint8_t* q, uint8_t* s,
              cudaStream_t st) {
  if (M < 0 || K <= 0) return BASAL200_ERR_ARG;
  if (K % 64) return BASAL200_ERR_SHAPE;
  if (M == 0) return BASAL200_OK;
  if (!x || !inv_g || !q || !s) return BASAL200_ERR_ARG;
  if (!aligned16(x) || !aligned16(q) || !aligned16(s)) return BASAL200_ERR_ALIGN;
  const int64_t Mp = (M + 127) / 128 * 128;
  if (Mp / 128 > 65535 || K / 64 > 65535) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t tiles = K / 64;
  // 2 tiles a CTA once that still gives every SM 4 CTAs
  const bool two = (tiles / 2) * (Mp / 128) >= (int64_t)g_dev[dev].sms * 4;
  const dim3 grid((unsigned)(two ? (tiles + 1) / 2 : tiles), (unsigned)(Mp / 128));
  const int early = early_trigger(dev, (int64_t)grid.x * grid.y, 1);
  switch (xt) {
    case BASAL200_BF16:
      return two ? launch_pdl(nvfp4_act_quant_kernel<__nv_bfloat16, 2>, grid, 512, 0, st,
                              static_cast<const __nv_bfloat16*>(x), inv_g, M, K, q, s, early)
                 : launch_pdl(nvfp4_act_quant_kernel<__nv_bfloat16, 1>, grid, 512, 0, st,
                              static_cast<const __nv_bfloat16*>(x), inv_g, M, K, q, s, early);
    case BASAL200_F16:
      return two ? launch_pdl(nvfp4_act_quant_kernel<__half, 2>, grid, 512, 0, st, static_cast<const __half*>(x),
                              inv_g, M, K, q, s, early)
                 : launch_pdl(nvfp4_act_quant_kernel<__half, 1>, grid, 512, 0, st, static_cast<const __half*>(x),
                              inv_g, M, K, q, s, early);
    case BASAL200_F32:
      return two ? launch_pdl(nvfp4_act_quant_kernel<float, 2>, grid, 512, 0, st, static_cast<const float*>(x), inv_g,
                              M, K, q, s, early)
                 : launch_pdl(nvfp4_act_quant_kernel<float, 1>, grid, 512, 0, st, static_cast<const float*>(x), inv_g,
                              M, K, q, s, early);
    default:
      return BASAL200_ERR_DTYPE;
  }
  return launched();
}

template <typename T>
int nvfp4_wq_typed(const T* w, int64_t N, int64_t K, uint8_t* codes, uint8_t* scales, float* g, int dev,
                   cudaStream_t st) {
  if (cudaMemsetAsync(g, 0, sizeof(float), st) != cudaSuccess) return BASAL200_ERR_LAUNCH;
  const int64_t n8 = N * K / 8;
  absmax_kernel<T><<<grid_for(dev, n8, 256), 256, 0, st>>>(w, n8, reinterpret_cast<unsigned*>(g));
  const int64_t Np = (N + 127) / 128 * 128, c4 = (K / 16 + 3) / 4;
  const int64_t blocks16 = Np * c4 * 4;
  if ((blocks16 + 255) / 256 > INT32_MAX) return BASAL200_ERR_LIMIT;
  nvfp4_weight_quant_kernel<T><<<(unsigned)((blocks16 + 255) / 256), 256, 0, st>>>(w, g, N, Np, K, c4, codes, scales);
  nvfp4_global_scale_kernel<<<1, 1, 0, st>>>(g);
  return launched();
}

// ------------------------------------------------------------------------------------------------------------
// GEMMs
// ------------------------------------------------------------------------------------------------------------

// The block GEMM moves registers between warpgroups (setmaxnreg); a launch with fewer registers a thread than the
// split needs would wait forever, so the compiled kernel's count is checked before its first launch on a device.
template <typename K>
int check_launch_regs(K kernel, int need) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, kernel) != cudaSuccess) return BASAL200_ERR_LAUNCH;
  if (a.numRegs < need) {
    fprintf(stderr, "libbasal200: kernel built with %d registers a thread, its register split needs %d\n", a.numRegs,
            need);
    return BASAL200_ERR_LAUNCH;
  }
  return BASAL200_OK;
}

template <bool INT8, int OUT, int ACT = blockgemm::kActNone, bool RES = false>
int block_gemm_launch(int dev, const CUtensorMap& ta, const CUtensorMap& tb, const blockgemm::OutMaps& out,
                      const blockgemm::Params& p, cudaStream_t st) {
  auto kern = blockgemm::block_gemm_kernel<INT8, OUT, ACT, RES>;
  const int slot = RES ? kSlotRes + (INT8 ? 2 : 0) + (OUT == BASAL200_F16 ? 1 : 0)
                       : ACT == blockgemm::kActNone
                             ? kSlotBlock + (INT8 ? 3 : 0) + OUT
                             : kSlotGlu + (INT8 ? 4 : 0) + (OUT == BASAL200_F16 ? 2 : 0) + ACT - 1;
  if (!smem_is_set(dev, slot)) {
    const int rc = check_launch_regs(kern, (int)blockgemm::LAUNCH_REGS);
    if (rc) return rc;
  }
  int rc = set_smem(dev, slot, kern, blockgemm::smem_bytes<OUT>());
  if (rc) return rc;
  const int grid = p.num_tiles < g_dev[dev].sms ? p.num_tiles : g_dev[dev].sms;
  return launch_pdl(kern, grid, blockgemm::NUM_THREADS, blockgemm::smem_bytes<OUT>(), st, ta, tb, out, p);
}

// Few rows (M <= 64): the weight-streaming kernel, NT token rows a tile (32 or 64), one CTA per 128-row weight tile.
template <bool INT8, int OUT, int NT>
int small_gemm_launch(int dev, const void* q, const float* s, const void* w, const float* ws, const void* bias,
                      void* const* cs, int npeers, int64_t ldc, int col_off, int64_t M, int64_t N, int64_t K,
                      cudaStream_t st, const uint32_t* gate = nullptr) {
  auto kern = smallgemm::small_gemm_kernel<INT8, OUT, NT>;
  constexpr size_t smem = smallgemm::smem_bytes<NT>();
  const int slot = kSlotSmall + (INT8 ? 6 : 0) + OUT * 2 + (NT == 32 ? 0 : 1);
  int rc = set_smem(dev, slot, kern, smem);
  if (rc) return rc;
  CUtensorMap tw, tt;
  if ((rc = tmap_u8(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, smallgemm::BK, smallgemm::BW))) return rc;
  if ((rc = tmap_u8(&tt, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, smallgemm::BK, NT))) return rc;
  smallgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = bias;
  for (int r = 0; r < blockgemm::kMaxPeers; ++r) p.cs[r] = r < npeers ? cs[r] : nullptr;
  p.npeers = npeers;
  p.ldc = ldc;
  p.col_off = col_off;
  p.M = (int)M;
  p.N = (int)N;
  p.nkb = (int)(K / 128);
  p.gate = gate;
  return launch_pdl(kern, (unsigned)(N / smallgemm::BW), smallgemm::Cfg<NT>::THREADS, smem, st, tw, tt, p);
}

template <bool INT8, int OUT>
int small_gemm(int dev, const void* q, const float* s, const void* w, const float* ws, const void* bias,
               void* const* cs, int npeers, int64_t ldc, int col_off, int64_t M, int64_t N, int64_t K,
               cudaStream_t st, const uint32_t* gate = nullptr) {
  if (M <= 32)
    return small_gemm_launch<INT8, OUT, 32>(dev, q, s, w, ws, bias, cs, npeers, ldc, col_off, M, N, K, st, gate);
  return small_gemm_launch<INT8, OUT, 64>(dev, q, s, w, ws, bias, cs, npeers, ldc, col_off, M, N, K, st, gate);
}

// Few rows and fewer weight tiles than this: the split kernels (every SM streams weights), when the caller's
// workspace holds the products and they stay well inside L2.
constexpr int64_t kSplitMaxTiles = 64;  // measured at N = 12288 (96 tiles): no faster than one CTA a tile
constexpr int64_t kSplitMaxBytes = (int64_t)32 << 20;

// Workspace bytes that make the few-rows GEMM of (M, N, K) take the split kernels; 0 for a shape that does not.
int64_t split_workspace(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > smallgemm::MAX_ROWS || N <= 0 || K <= 0 || N % 128 || K % 128) return 0;
  const int64_t tiles = N / smallgemm::BW, nkb = K / 128;
  if (nkb < 2 || nkb > smallgemm::MAX_KB || tiles > kSplitMaxTiles) return 0;
  const int64_t bytes = smallgemm::split_prod_bytes(M, N, nkb);
  return bytes <= kSplitMaxBytes ? bytes : 0;
}

// TX = void: q holds the activation codes (TMA-loaded). TX = __nv_bfloat16 / __half: the fused linear, q is the
// activations themselves, quantised inside the products kernel, and their scales are written to s.
template <bool INT8, int OUT, int NT, typename TX>
int split_gemm_launch(int dev, const void* q, const float* s, const void* w, const float* ws, const void* bias,
                      void* const* cs, int npeers, int64_t ldc, int col_off, int64_t M, int64_t N, int64_t K,
                      void* work, cudaStream_t st) {
  constexpr bool QUANT = !std::is_void<TX>::value;
  auto kp = smallgemm::split_products_kernel<INT8, NT, TX>;
  constexpr size_t smem = smallgemm::split_smem_bytes<NT>();
  const int slot = (QUANT ? kSlotSplitQ + (std::is_same<TX, __half>::value ? 4 : 0) : kSlotSplit) + (INT8 ? 2 : 0) +
                   (NT == 32 ? 0 : 1);
  int rc = set_smem(dev, slot, kp, smem);
  if (rc) return rc;
  CUtensorMap tw, tt;
  if ((rc = tmap_u8(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, smallgemm::BK, smallgemm::BW))) return rc;
  if (QUANT)
    tt = tw;  // unused: the tokens are quantised in the kernel
  else if ((rc = tmap_u8(&tt, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, smallgemm::BK, NT)))
    return rc;
  smallgemm::SplitParams sp;
  sp.prod = static_cast<float*>(work);
  sp.M = (int)M;
  sp.nkb = (int)(K / 128);
  sp.units = N / smallgemm::BW * sp.nkb;
  sp.x = QUANT ? q : nullptr;
  sp.s = QUANT ? const_cast<float*>(s) : nullptr;
  const int64_t grid = sp.units < g_dev[dev].sms ? sp.units : g_dev[dev].sms;
  constexpr int threads = smallgemm::split_threads<NT, TX>();
  if ((rc = launch_pdl(kp, (unsigned)grid, threads, smem, st, tw, tt, sp))) return rc;
  smallgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = bias;
  for (int r = 0; r < blockgemm::kMaxPeers; ++r) p.cs[r] = r < npeers ? cs[r] : nullptr;
  p.npeers = npeers;
  p.ldc = ldc;
  p.col_off = col_off;
  p.M = (int)M;
  p.N = (int)N;
  p.nkb = sp.nkb;
  const dim3 rgrid((unsigned)(N / smallgemm::BW), (unsigned)M);
  return launch_pdl(smallgemm::split_reduce_kernel<OUT>, rgrid, smallgemm::REDUCE_THREADS, 0, st,
                    static_cast<const float*>(work), p);
}

template <bool INT8, int OUT, typename TX = void>
int split_gemm(int dev, const void* q, const float* s, const void* w, const float* ws, const void* bias, void* c,
               int64_t M, int64_t N, int64_t K, void* work, cudaStream_t st) {
  void* const cs[1] = {c};
  if (M <= 32) return split_gemm_launch<INT8, OUT, 32, TX>(dev, q, s, w, ws, bias, cs, 1, N, 0, M, N, K, work, st);
  return split_gemm_launch<INT8, OUT, 64, TX>(dev, q, s, w, ws, bias, cs, 1, N, 0, M, N, K, work, st);
}

// The few-rows linear with the activation quantiser fused into the split GEMM (16-bit x, output in x's type): one
// launch fewer than act_quant + GEMM, the same codes, scales and output bits. Returns -1 when it does not apply.
template <bool INT8>
int fused_split_linear(const void* x, int xt, const void* w, const float* ws, const void* bias, void* y,
                       int64_t M, int64_t N, int64_t K, float* s_scratch, void* work, int64_t work_bytes,
                       cudaStream_t st) {
  if (xt != BASAL200_BF16 && xt != BASAL200_F16) return -1;
  if (M < 1 || K <= 0 || K % 128 || N % 128) return -1;
  const int64_t split = split_workspace(M, N, K);
  if (split <= 0 || !work || work_bytes < split) return -1;
  if (!x || !w || !ws || !y || !s_scratch) return BASAL200_ERR_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || !aligned16(work) || (bias && !aligned16(bias)))
    return BASAL200_ERR_ALIGN;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  if (xt == BASAL200_BF16)
    return split_gemm<INT8, BASAL200_BF16, __nv_bfloat16>(dev, x, s_scratch, w, ws, bias, y, M, N, K, work, st);
  return split_gemm<INT8, BASAL200_F16, __half>(dev, x, s_scratch, w, ws, bias, y, M, N, K, work, st);
}

// work / work_bytes: the caller's workspace (may be null); when it holds split_workspace(M, N, K) > 0 bytes, the
// few-rows GEMM runs split over the SMs, otherwise unsplit (the same bits either way).
template <bool INT8>
int block_gemm(const void* q, const float* s, const void* w, const float* ws, const void* bias, void* c, int ct,
               int64_t M, int64_t N, int64_t K, void* work, int64_t work_bytes, cudaStream_t st) {
  if (M < 0 || N <= 0 || K <= 0) return BASAL200_ERR_ARG;
  if (N % 128 || K % 128) return BASAL200_ERR_SHAPE;
  if (M == 0) return BASAL200_OK;
  if (!q || !s || !w || !ws || !c) return BASAL200_ERR_ARG;
  if (!aligned16(q) || !aligned16(w) || !aligned16(c) || (bias && !aligned16(bias))) return BASAL200_ERR_ALIGN;
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  void* const cs[1] = {c};
  const int64_t split = split_workspace(M, N, K);
  if (split > 0 && work && work_bytes >= split) {
    if (!aligned16(work)) return BASAL200_ERR_ALIGN;
    switch (ct) {
      case BASAL200_BF16: return split_gemm<INT8, BASAL200_BF16>(dev, q, s, w, ws, bias, c, M, N, K, work, st);
      case BASAL200_F16: return split_gemm<INT8, BASAL200_F16>(dev, q, s, w, ws, bias, c, M, N, K, work, st);
      case BASAL200_F32: return split_gemm<INT8, BASAL200_F32>(dev, q, s, w, ws, bias, c, M, N, K, work, st);
      default: return BASAL200_ERR_DTYPE;
    }
  }
  if (M <= smallgemm::MAX_ROWS && K / 128 <= smallgemm::MAX_KB && N / smallgemm::BW <= 65535) {
    switch (ct) {
      case BASAL200_BF16: return small_gemm<INT8, BASAL200_BF16>(dev, q, s, w, ws, bias, cs, 1, N, 0, M, N, K, st);
      case BASAL200_F16: return small_gemm<INT8, BASAL200_F16>(dev, q, s, w, ws, bias, cs, 1, N, 0, M, N, K, st);
      case BASAL200_F32: return small_gemm<INT8, BASAL200_F32>(dev, q, s, w, ws, bias, cs, 1, N, 0, M, N, K, st);
      default: return BASAL200_ERR_DTYPE;
    }
  }
  CUtensorMap ta, tb;
  blockgemm::OutMaps out;
  memset(&out, 0, sizeof(out));
  if ((rc = tmap_u8(&ta, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, blockgemm::BK, blockgemm::BM))) return rc;
  if ((rc = tmap_u8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, blockgemm::BK, blockgemm::BN))) return rc;
  // fp32 outputs are stored directly, without TMA
  if (ct != BASAL200_F32 && (rc = tmap_u16(&out.m[0], c, (uint64_t)N, (uint64_t)M, 64, blockgemm::BM))) return rc;
  blockgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = bias;
  p.c = c;
  p.M = (int)M;
  p.N = (int)N;
  p.nkb = (int)(K / 128);
  p.tiles_n = (int)((N + blockgemm::BN - 1) / blockgemm::BN);
  p.npeers = 1;
  p.col_off = 0;
  p.glu_up = 0;
  const int64_t tiles = (M + blockgemm::BM - 1) / blockgemm::BM * p.tiles_n;
  if (tiles > INT32_MAX) return BASAL200_ERR_LIMIT;
  p.num_tiles = (int)tiles;
  switch (ct) {
    case BASAL200_BF16: return block_gemm_launch<INT8, BASAL200_BF16>(dev, ta, tb, out, p, st);
    case BASAL200_F16: return block_gemm_launch<INT8, BASAL200_F16>(dev, ta, tb, out, p, st);
    case BASAL200_F32: return block_gemm_launch<INT8, BASAL200_F32>(dev, ta, tb, out, p, st);
    default: return BASAL200_ERR_DTYPE;
  }
}

// The FP8 block GEMM of one rank's column shard of a column-parallel linear (N of n_total weight rows, from column
// col_off), its tiles stored into every rank's [M, n_total] output (outs: npeers device pointers, peer-mapped):
// the linear's all-gather done by the GEMM's own stores, tile by tile, with no collective kernel. 16-bit outputs.
// pad: this rank's peer-barrier pad (or null); when its status word is set, the kernel stores nothing.
int block_gemm_gather(const void* q, const float* s, const void* w, const float* ws, void* const* outs, int npeers,
                      int64_t col_off, int64_t n_total, int ct, int64_t M, int64_t N, int64_t K, const uint32_t* pad,
                      cudaStream_t st) {
  if (M < 0 || N <= 0 || K <= 0 || npeers < 1 || npeers > blockgemm::kMaxPeers || !outs) return BASAL200_ERR_ARG;
  if (N % 128 || K % 128 || col_off % 128 || col_off + N > n_total) return BASAL200_ERR_SHAPE;
  if (ct != BASAL200_BF16 && ct != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (M == 0) return BASAL200_OK;
  if (!q || !s || !w || !ws) return BASAL200_ERR_ARG;
  if (!aligned16(q) || !aligned16(w)) return BASAL200_ERR_ALIGN;
  for (int r = 0; r < npeers; ++r)
    if (!outs[r] || !aligned16(outs[r])) return BASAL200_ERR_ALIGN;
  if (M > (int64_t)1 << 30 || n_total > (int64_t)1 << 30) return BASAL200_ERR_LIMIT;
  if (pad && (reinterpret_cast<uintptr_t>(pad) & 3)) return BASAL200_ERR_ALIGN;
  static_assert(blockgemm::kPadStatus == BASAL200_PAD_STATUS_WORD, "the pad layout of include/basal200.h");
  const uint32_t* gate = pad ? pad + blockgemm::kPadStatus : nullptr;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  if (M <= smallgemm::MAX_ROWS && K / 128 <= smallgemm::MAX_KB && N / smallgemm::BW <= 65535) {
    if (ct == BASAL200_BF16)
      return small_gemm<false, BASAL200_BF16>(dev, q, s, w, ws, nullptr, outs, npeers, n_total, (int)col_off, M, N, K,
                                              st, gate);
    return small_gemm<false, BASAL200_F16>(dev, q, s, w, ws, nullptr, outs, npeers, n_total, (int)col_off, M, N, K,
                                           st, gate);
  }
  CUtensorMap ta, tb;
  blockgemm::OutMaps out;
  memset(&out, 0, sizeof(out));
  if ((rc = tmap_u8(&ta, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, blockgemm::BK, blockgemm::BM))) return rc;
  if ((rc = tmap_u8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, blockgemm::BK, blockgemm::BN))) return rc;
  for (int r = 0; r < npeers; ++r)
    if ((rc = tmap_u16(&out.m[r], outs[r], (uint64_t)n_total, (uint64_t)M, 64, blockgemm::BM))) return rc;
  blockgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = nullptr;
  p.c = nullptr;
  p.M = (int)M;
  p.N = (int)N;
  p.nkb = (int)(K / 128);
  p.tiles_n = (int)((N + blockgemm::BN - 1) / blockgemm::BN);
  p.npeers = npeers;
  p.col_off = (int)col_off;
  p.glu_up = 0;
  p.gate = gate;
  const int64_t tiles = (M + blockgemm::BM - 1) / blockgemm::BM * p.tiles_n;
  if (tiles > INT32_MAX) return BASAL200_ERR_LIMIT;
  p.num_tiles = (int)tiles;
  if (ct == BASAL200_BF16) return block_gemm_launch<false, BASAL200_BF16>(dev, ta, tb, out, p, st);
  return block_gemm_launch<false, BASAL200_F16>(dev, ta, tb, out, p, st);
}

template <int OUT, int BN>
int fp4_gemm_launch(int dev, const void* q, const void* w, int64_t Mp, int64_t N, int64_t K, fp4gemm::Params p,
                    cudaStream_t st) {
  CUtensorMap ta, tb;
  int rc;
  // the activation map ends at row M: the TMA fills the rows of the last 128-row tile past M with zero codes (the
  // bytes the quantiser wrote there) without reading them, which matters for few rows (M = 16: 16 of 128 rows)
  if ((rc = tmap_u8(&ta, q, (uint64_t)(K / 2), (uint64_t)p.M, (uint64_t)(K / 2), fp4gemm::BKB, fp4gemm::BM)))
    return rc;
  if ((rc = tmap_u8(&tb, w, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), fp4gemm::BKB, BN))) return rc;
  p.tiles_n = (int)((N + BN - 1) / BN);
  const int64_t tiles = Mp / fp4gemm::BM * p.tiles_n;
  if (tiles > INT32_MAX) return BASAL200_ERR_LIMIT;
  p.num_tiles = (int)tiles;
  auto kern = fp4gemm::nvfp4_gemm_kernel<OUT, BN>;
  constexpr size_t smem = fp4gemm::Cfg<BN>::SMEM_BYTES;
  if ((rc = set_smem(dev, kSlotFp4 + OUT * 2 + (BN == 256 ? 0 : 1), kern, smem))) return rc;
  const int grid = p.num_tiles < g_dev[dev].sms ? p.num_tiles : g_dev[dev].sms;
  return launch_pdl(kern, grid, fp4gemm::NUM_THREADS, smem, st, ta, tb, p);
}

// 128 x 256 tiles, or 128 x 128 when the wide tiles would not give every SM one (few rows)
template <int OUT>
int fp4_gemm_pick(int dev, const void* q, const void* w, int64_t Mp, int64_t N, int64_t K, const fp4gemm::Params& p,
                  cudaStream_t st) {
  if (Mp / fp4gemm::BM * ((N + 255) / 256) < g_dev[dev].sms)
    return fp4_gemm_launch<OUT, 128>(dev, q, w, Mp, N, K, p, st);
  return fp4_gemm_launch<OUT, 256>(dev, q, w, Mp, N, K, p, st);
}

int fp4_gemm(const uint8_t* q, const uint8_t* s, const uint8_t* w, const uint8_t* ws, const float* alpha,
             const void* bias, void* y, int yt, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  if (M < 0 || N <= 0 || K <= 0) return BASAL200_ERR_ARG;
  if (K % 64 || N % 16) return BASAL200_ERR_SHAPE;
  if (M == 0) return BASAL200_OK;
  if (!q || !s || !w || !ws || !alpha || !y) return BASAL200_ERR_ARG;
  if (!aligned16(q) || !aligned16(s) || !aligned16(w) || !aligned16(ws) || !aligned16(y) ||
      (bias && !aligned16(bias)))
    return BASAL200_ERR_ALIGN;
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t Mp = (M + 127) / 128 * 128;
  fp4gemm::Params p;
  p.sa = s;
  p.sb = ws;
  p.alpha = alpha;
  p.bias = bias;
  p.y = y;
  p.M = (int)M;
  p.N = (int)N;
  p.nchunk = (int)(K / 64);
  p.nkb = (p.nchunk + 3) / 4;
  p.nblk_b = (int)((N + 127) / 128);
  switch (yt) {
    case BASAL200_BF16: return fp4_gemm_pick<BASAL200_BF16>(dev, q, w, Mp, N, K, p, st);
    case BASAL200_F16: return fp4_gemm_pick<BASAL200_F16>(dev, q, w, Mp, N, K, p, st);
    case BASAL200_F32: return fp4_gemm_pick<BASAL200_F32>(dev, q, w, Mp, N, K, p, st);
    default: return BASAL200_ERR_DTYPE;
  }
}

// ------------------------------------------------------------------------------------------------------------
// readout
// ------------------------------------------------------------------------------------------------------------
// code_logits: the warp-item kernel with CW codes an item (4, 8 or 16: the fewest that cover U, up to 16).
template <typename T>
constexpr int type_index() {
  return std::is_same<T, float>::value ? 0 : (std::is_same<T, __nv_bfloat16>::value ? 1 : 2);
}

// The tensor-core kernel: a cluster of 8 CTAs (one per feature slice) on each tile of 128 prompts x BN codes.
template <typename T, typename TB, int BN>
int logits_tc_launch(int dev, const T* h, int64_t R, int64_t D, int64_t ldh, const T* head, int64_t V, int64_t ldw,
                     const int64_t* ids, int64_t U, const TB* bias, float softcap, float* z, cudaStream_t st) {
  auto kern = readout::code_logits_tc_kernel<T, TB, BN>;
  constexpr size_t smem = readout::tc_smem_bytes<BN>();
  const int slot = kSlotLogitsTc + (std::is_same<T, __half>::value ? 6 : 0) + type_index<TB>() * 2 + (BN == 32);
  int rc = set_smem(dev, slot, kern, smem);
  if (rc) return rc;
  const int64_t gx = (R + readout::TM - 1) / readout::TM, gy = (U + BN - 1) / BN;
  if (gx > INT32_MAX || gy > 65535) return BASAL200_ERR_LIMIT;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = readout::TSPLIT;
  cfg.gridDim = dim3((unsigned)gx, (unsigned)gy, readout::TSPLIT);
  cfg.blockDim = readout::TTHREADS;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, h, R, D, ldh, head, V, ldw, ids, U, bias, softcap, z) != cudaSuccess)
    return launched();
  return launched();
}

template <typename TH, typename TW, typename TB>
int logits_launch(int dev, const TH* h, int64_t R, int64_t D, int64_t ldh, const TW* head, int64_t V, int64_t ldw,
                  const int64_t* ids, int64_t U, const TB* bias, float softcap, float* z, cudaStream_t st) {
  if constexpr (std::is_same<TH, TW>::value && sizeof(TH) == 2) {
    // one 16-bit type, 16-byte aligned rows, D % 8 == 0: the tensor cores, whatever R and U (so a logit's bits never
    // depend on them)
    if (D % 8 == 0 && aligned16(h) && aligned16(head) && ldh % 8 == 0 && ldw % 8 == 0) {
      if (U <= 16) return logits_tc_launch<TH, TB, 16>(dev, h, R, D, ldh, head, V, ldw, ids, U, bias, softcap, z, st);
      return logits_tc_launch<TH, TB, 32>(dev, h, R, D, ldh, head, V, ldw, ids, U, bias, softcap, z, st);
    }
  }
  if constexpr (sizeof(TH) == 2 && sizeof(TW) == 2) {
    // many codes, whole 256-feature chunks, 16-byte aligned rows: the staged kernel (the same bits)
    if (U > 8 && D % readout::CHUNK == 0 && aligned16(h) && aligned16(head) && (ldh * 2) % 16 == 0 &&
        (ldw * 2) % 16 == 0) {
      auto kern = readout::code_logits_staged_kernel<TH, TW, TB>;
      constexpr size_t smem = sizeof(readout::StagedSmem<TH, TW>);
      const int slot = kSlotLogits + (type_index<TH>() - 1) * 6 + (type_index<TW>() - 1) * 3 + type_index<TB>();
      int rc = set_smem(dev, slot, kern, smem);
      if (rc) return rc;
      const int64_t gy = (R + readout::SR - 1) / readout::SR;
      if (gy > 65535) return BASAL200_ERR_LIMIT;
      const dim3 grid((unsigned)((U + readout::SU - 1) / readout::SU), (unsigned)gy);
      return launch_pdl(kern, grid, readout::SWARPS * 32, smem, st, h, R, D, ldh, head, V, ldw, ids, U, bias, softcap,
                        z);
    }
  }
  const int cw = U <= 4 ? 4 : (U <= 8 ? 8 : 16);
  const int64_t items = (R + readout::PW - 1) / readout::PW * ((U + cw - 1) / cw);
  const int64_t grid = (items + readout::IWARPS - 1) / readout::IWARPS;
  if (grid > INT32_MAX) return BASAL200_ERR_LIMIT;
  constexpr int threads = readout::IWARPS * 32;
  if (cw == 4)
    return launch_pdl(readout::code_logits_warp_kernel<TH, TW, TB, 4>, (unsigned)grid, threads, 0, st, h, R, D, ldh,
                      head, V, ldw, ids, U, bias, softcap, z);
  if (cw == 8)
    return launch_pdl(readout::code_logits_warp_kernel<TH, TW, TB, 8>, (unsigned)grid, threads, 0, st, h, R, D, ldh,
                      head, V, ldw, ids, U, bias, softcap, z);
  return launch_pdl(readout::code_logits_warp_kernel<TH, TW, TB, 16>, (unsigned)grid, threads, 0, st, h, R, D, ldh,
                    head, V, ldw, ids, U, bias, softcap, z);
}

template <typename TH, typename TW>
int logits_typed(int dev, const TH* h, int64_t R, int64_t D, int64_t ldh, const TW* head, int64_t V, int64_t ldw,
                 const int64_t* ids, int64_t U, const void* bias, int bt, float softcap, float* z, cudaStream_t st) {
  if (!bias)
    return logits_launch(dev, h, R, D, ldh, head, V, ldw, ids, U, static_cast<const float*>(nullptr), softcap, z, st);
  if (bt == BASAL200_F32)
    return logits_launch(dev, h, R, D, ldh, head, V, ldw, ids, U, static_cast<const float*>(bias), softcap, z, st);
  if (bt == BASAL200_BF16)
    return logits_launch(dev, h, R, D, ldh, head, V, ldw, ids, U, static_cast<const __nv_bfloat16*>(bias), softcap,
                         z, st);
  if (bt == BASAL200_F16)
    return logits_launch(dev, h, R, D, ldh, head, V, ldw, ids, U, static_cast<const __half*>(bias), softcap, z, st);
  return BASAL200_ERR_DTYPE;
}

template <typename TH>
int logits_head(int dev, const TH* h, int64_t R, int64_t D, int64_t ldh, const void* head, int ht, int64_t V,
                int64_t ldw, const int64_t* ids, int64_t U, const void* bias, int bt, float softcap, float* z,
                cudaStream_t st) {
  switch (ht) {
    case BASAL200_BF16:
      return logits_typed(dev, h, R, D, ldh, static_cast<const __nv_bfloat16*>(head), V, ldw, ids, U, bias, bt, softcap,
                          z, st);
    case BASAL200_F16:
      return logits_typed(dev, h, R, D, ldh, static_cast<const __half*>(head), V, ldw, ids, U, bias, bt, softcap, z,
                          st);
    case BASAL200_F32:
      return logits_typed(dev, h, R, D, ldh, static_cast<const float*>(head), V, ldw, ids, U, bias, bt, softcap, z, st);
    default:
      return BASAL200_ERR_DTYPE;
  }
}

}  // namespace

// The gated linear y = act(x W_gate^T) * (x W_up^T) of a merged block-quantised [gate; up] weight w [2I, K]: the
// activation quantiser, then the block GEMM whose epilogue pairs gate block n with up block n (any M: the many-rows
// kernel; rows past M are clipped by the tensor maps).
template <bool INT8, int OUT>
int glu_launch(int dev, const CUtensorMap& ta, const CUtensorMap& tb, const blockgemm::OutMaps& out,
               const blockgemm::Params& p, int act, cudaStream_t st) {
  if (act == BASAL200_ACT_SILU) return block_gemm_launch<INT8, OUT, blockgemm::kActSilu>(dev, ta, tb, out, p, st);
  return block_gemm_launch<INT8, OUT, blockgemm::kActGeluTanh>(dev, ta, tb, out, p, st);
}

// Few rows: the merged linear into a [M, 2I] temporary of the workspace (few-rows or split kernels, the same bits as
// the gated epilogue's gate and up values), then glu_rows_kernel.
int64_t glu_temp_bytes(int64_t M, int64_t I) { return (M * 2 * I * 2 + 255) / 256 * 256; }
int64_t glu_workspace(int64_t M, int64_t I, int64_t K) {
  if (M < 1 || M > smallgemm::MAX_ROWS || I <= 0 || K <= 0 || I % 128 || K % 128) return 0;
  return glu_temp_bytes(M, I) + split_workspace(M, 2 * I, K);
}

template <int OUT>
int glu_rows_launch(const void* t, void* y, int64_t M, int64_t I, int act, cudaStream_t st) {
  const int64_t grid = (M * I / 8 + 255) / 256;
  if (act == BASAL200_ACT_SILU)
    return launch_pdl(blockgemm::glu_rows_kernel<OUT, blockgemm::kActSilu>, (unsigned)grid, 256, 0, st, t, y, M, I);
  return launch_pdl(blockgemm::glu_rows_kernel<OUT, blockgemm::kActGeluTanh>, (unsigned)grid, 256, 0, st, t, y, M,
                    I);
}

// codes: q / s already hold x's activation codes and scales (the entry points that take codes); x is not read.
template <bool INT8>
int block_linear_glu(const void* x, int xt, const void* w, const float* ws, void* y, int64_t M, int64_t I, int64_t K,
                     int act, void* q, float* s, void* work, int64_t work_bytes, cudaStream_t st, bool codes = false) {
  if (M < 0 || I <= 0 || K <= 0) return BASAL200_ERR_ARG;
  if (act != BASAL200_ACT_SILU && act != BASAL200_ACT_GELU_TANH) return BASAL200_ERR_ARG;
  if (I % 128 || K % 128) return BASAL200_ERR_SHAPE;
  if (xt != BASAL200_BF16 && xt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (M == 0) return BASAL200_OK;
  if ((!x && !codes) || !w || !ws || !y || !q || !s) return BASAL200_ERR_ARG;
  if (!aligned16(w) || !aligned16(y) || !aligned16(q)) return BASAL200_ERR_ALIGN;
  if (M > (int64_t)1 << 30 || I > (int64_t)1 << 29) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t need = glu_workspace(M, I, K);
  if (need > 0 && work && work_bytes >= need) {  // few rows
    if (!aligned16(work)) return BASAL200_ERR_ALIGN;
    uint8_t* temp = static_cast<uint8_t*>(work);
    uint8_t* split = temp + glu_temp_bytes(M, I);
    const int64_t split_bytes = work_bytes - glu_temp_bytes(M, I);
    if (codes)
      rc = block_gemm<INT8>(q, s, w, ws, nullptr, temp, xt, M, 2 * I, K, split, split_bytes, st);
    else if (INT8)
      rc = basal200_int8_block_linear(x, xt, static_cast<const int8_t*>(w), ws, nullptr, temp, M, 2 * I, K,
                                      static_cast<int8_t*>(q), s, split, split_bytes, st);
    else
      rc = basal200_fp8_block_linear(x, xt, static_cast<const uint8_t*>(w), ws, nullptr, temp, M, 2 * I, K,
                                     static_cast<uint8_t*>(q), s, split, split_bytes, st);
    if (rc) return rc;
    return xt == BASAL200_BF16 ? glu_rows_launch<BASAL200_BF16>(temp, y, M, I, act, st)
                               : glu_rows_launch<BASAL200_F16>(temp, y, M, I, act, st);
  }
  if (!codes && (rc = act_quant<INT8>(x, xt, M, K, q, s, st))) return rc;
  CUtensorMap ta, tb;
  blockgemm::OutMaps out;
  memset(&out, 0, sizeof(out));
  if ((rc = tmap_u8(&ta, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, blockgemm::BK, blockgemm::BM))) return rc;
  if ((rc = tmap_u8(&tb, w, (uint64_t)K, (uint64_t)(2 * I), (uint64_t)K, blockgemm::BK, 128))) return rc;
  if ((rc = tmap_u16(&out.m[0], y, (uint64_t)I, (uint64_t)M, 64, blockgemm::BM))) return rc;
  blockgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = nullptr;
  p.c = nullptr;
  p.M = (int)M;
  p.N = (int)I;
  p.nkb = (int)(K / 128);
  p.tiles_n = (int)(I / 128);
  p.npeers = 1;
  p.col_off = 0;
  p.glu_up = (int)I;
  const int64_t tiles = (M + blockgemm::BM - 1) / blockgemm::BM * p.tiles_n;
  if (tiles > INT32_MAX) return BASAL200_ERR_LIMIT;
  p.num_tiles = (int)tiles;
  if (xt == BASAL200_BF16) return glu_launch<INT8, BASAL200_BF16>(dev, ta, tb, out, p, act, st);
  return glu_launch<INT8, BASAL200_F16>(dev, ta, tb, out, p, act, st);
}

// The linear with the residual added in the epilogue: y = residual + linear(x) (+ bias), both 16-bit, with torch's
// roundings (the linear's output cast, the sum cast). Many rows: the block GEMM whose epilogue loads the residual
// tile; few rows with the workspace: the few-rows / split linear into a temporary, then add_rows_kernel (same bits).
int64_t res_temp_bytes(int64_t M, int64_t N) { return (M * N * 2 + 255) / 256 * 256; }
int64_t res_workspace(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > smallgemm::MAX_ROWS || N <= 0 || K <= 0 || N % 128 || K % 128) return 0;
  return res_temp_bytes(M, N) + split_workspace(M, N, K);
}

template <bool INT8>
int block_linear_residual(const void* x, int xt, const void* w, const float* ws, const void* bias, const void* res,
                          void* y, int64_t M, int64_t N, int64_t K, void* q, float* s, void* work, int64_t work_bytes,
                          cudaStream_t st, bool codes = false) {
  if (M < 0 || N <= 0 || K <= 0) return BASAL200_ERR_ARG;
  if (N % 128 || K % 128) return BASAL200_ERR_SHAPE;
  if (xt != BASAL200_BF16 && xt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (M == 0) return BASAL200_OK;
  if ((!x && !codes) || !w || !ws || !res || !y || !q || !s) return BASAL200_ERR_ARG;
  if (!aligned16(w) || !aligned16(y) || !aligned16(res) || !aligned16(q) || (bias && !aligned16(bias)))
    return BASAL200_ERR_ALIGN;
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t need = res_workspace(M, N, K);
  if (need > 0 && work && work_bytes >= need) {  // few rows
    if (!aligned16(work)) return BASAL200_ERR_ALIGN;
    uint8_t* temp = static_cast<uint8_t*>(work);
    uint8_t* split = temp + res_temp_bytes(M, N);
    const int64_t split_bytes = work_bytes - res_temp_bytes(M, N);
    if (codes)
      rc = block_gemm<INT8>(q, s, w, ws, bias, temp, xt, M, N, K, split, split_bytes, st);
    else if (INT8)
      rc = basal200_int8_block_linear(x, xt, static_cast<const int8_t*>(w), ws, bias, temp, M, N, K,
                                      static_cast<int8_t*>(q), s, split, split_bytes, st);
    else
      rc = basal200_fp8_block_linear(x, xt, static_cast<const uint8_t*>(w), ws, bias, temp, M, N, K,
                                     static_cast<uint8_t*>(q), s, split, split_bytes, st);
    if (rc) return rc;
    const int64_t grid = (M * N / 8 + 255) / 256;
    if (xt == BASAL200_BF16)
      return launch_pdl(blockgemm::add_rows_kernel<BASAL200_BF16>, (unsigned)grid, 256, 0, st,
                        static_cast<const void*>(temp), res, y, M * N);
    return launch_pdl(blockgemm::add_rows_kernel<BASAL200_F16>, (unsigned)grid, 256, 0, st,
                      static_cast<const void*>(temp), res, y, M * N);
  }
  if (!codes && (rc = act_quant<INT8>(x, xt, M, K, q, s, st))) return rc;
  CUtensorMap ta, tb;
  blockgemm::OutMaps out;
  memset(&out, 0, sizeof(out));
  if ((rc = tmap_u8(&ta, q, (uint64_t)K, (uint64_t)M, (uint64_t)K, blockgemm::BK, blockgemm::BM))) return rc;
  if ((rc = tmap_u8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, blockgemm::BK, blockgemm::BN))) return rc;
  if ((rc = tmap_u16(&out.m[0], y, (uint64_t)N, (uint64_t)M, 64, blockgemm::BM))) return rc;
  if ((rc = tmap_u16(&out.m[1], res, (uint64_t)N, (uint64_t)M, 64, blockgemm::BM))) return rc;
  blockgemm::Params p;
  p.s = s;
  p.ws = ws;
  p.bias = bias;
  p.c = nullptr;
  p.M = (int)M;
  p.N = (int)N;
  p.nkb = (int)(K / 128);
  p.tiles_n = (int)((N + blockgemm::BN - 1) / blockgemm::BN);
  p.npeers = 1;
  p.col_off = 0;
  p.glu_up = 0;
  const int64_t tiles = (M + blockgemm::BM - 1) / blockgemm::BM * p.tiles_n;
  if (tiles > INT32_MAX) return BASAL200_ERR_LIMIT;
  p.num_tiles = (int)tiles;
  if (xt == BASAL200_BF16)
    return block_gemm_launch<INT8, BASAL200_BF16, blockgemm::kActNone, true>(dev, ta, tb, out, p, st);
  return block_gemm_launch<INT8, BASAL200_F16, blockgemm::kActNone, true>(dev, ta, tb, out, p, st);
}

// ------------------------------------------------------------------------------------------------------------
// The config-5 hybrid decoder's element-wise steps (hybrid.cuh)
// ------------------------------------------------------------------------------------------------------------
int rms_quant(const void* x, int xt, const void* w, float eps, int64_t M, int64_t D, void* y, uint8_t* q, float* s,
              cudaStream_t st) {
  if (M < 0 || D <= 0 || !(eps >= 0.0f)) return BASAL200_ERR_ARG;
  if (D % 128) return BASAL200_ERR_SHAPE;
  if (xt != BASAL200_BF16 && xt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (M == 0) return BASAL200_OK;
  if (!x || !w || !q || !s) return BASAL200_ERR_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(q) || (y && !aligned16(y)) || (reinterpret_cast<uintptr_t>(s) & 3))
    return BASAL200_ERR_ALIGN;
  if (D > ((int64_t)1 << 20) || M > ((int64_t)1 << 34)) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const int64_t grid = (M + 7) / 8;  // a warp per row, 8 a CTA
  if (grid > INT32_MAX) return BASAL200_ERR_LIMIT;
  if (xt == BASAL200_BF16)
    return launch_pdl(hybrid::rms_quant_kernel<__nv_bfloat16>, (unsigned)grid, 256, 0, st,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), eps, M, (int)D,
                      static_cast<__nv_bfloat16*>(y), q, s);
  return launch_pdl(hybrid::rms_quant_kernel<__half>, (unsigned)grid, 256, 0, st, static_cast<const __half*>(x),
                    static_cast<const __half*>(w), eps, M, (int)D, static_cast<__half*>(y), q, s);
}

int gdn_prep(const void* proj, int dt, int64_t ld, const void* tail, int tail_rows, const void* conv, int kw,
             const float* A_log, const void* dt_bias, int b_off, int a_off, int rows, int T, int Hk, int Hv, float* q,
             float* k, void* v, float* beta, float* g, cudaStream_t st) {
  if (rows < 0 || T < 0 || Hk <= 0 || Hv <= 0 || kw < 1) return BASAL200_ERR_ARG;
  if (Hv % Hk || kw != 4) return BASAL200_ERR_SHAPE;  // the kernel's convolution has 4 taps (Qwen 3.5's)
  if (dt != BASAL200_BF16 && dt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (rows == 0 || T == 0) return BASAL200_OK;
  if (!proj || !conv || !A_log || !dt_bias || !q || !k || !v || !beta || !g) return BASAL200_ERR_ARG;
  if (tail && tail_rows != 1 && tail_rows != rows) return BASAL200_ERR_ARG;
  const int64_t C = (int64_t)(2 * Hk + Hv) * 128;
  if (ld < C || b_off < 0 || a_off < 0 || b_off + Hv > ld || a_off + Hv > ld) return BASAL200_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || (reinterpret_cast<uintptr_t>(v) & 7) || !aligned16(conv) || (ld % 4) ||
      (reinterpret_cast<uintptr_t>(proj) & 7) || (tail && (reinterpret_cast<uintptr_t>(tail) & 7)))
    return BASAL200_ERR_ALIGN;  // 8-byte loads of 4 channels, 16-byte loads of 4 channels' weights
  const int64_t items = (int64_t)rows * Hk * ((T + hybrid::PTB - 1) / hybrid::PTB);  // a warp each, 8 a CTA
  if ((items + 7) / 8 > INT32_MAX) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  hybrid::PrepParams p;
  p.proj = proj;
  p.ld = ld;
  p.tail = tail;
  p.tail_rows = tail_rows;
  p.conv = conv;
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  p.b_off = b_off;
  p.a_off = a_off;
  p.rows = rows;
  p.T = T;
  p.Hk = Hk;
  p.Hv = Hv;
  p.q_scale = 0.08838834764831845f;  // 128^-1/2, rounded to fp32 as torch rounds the Python float
  p.q = q;
  p.k = k;
  p.v = v;
  p.beta = beta;
  p.g = g;
  const unsigned grid = (unsigned)((items + 7) / 8);
  if (dt == BASAL200_BF16) return launch_pdl(hybrid::gdn_prep_kernel<__nv_bfloat16>, grid, 256, 0, st, p);
  return launch_pdl(hybrid::gdn_prep_kernel<__half>, grid, 256, 0, st, p);
}

template <typename T, typename TO>
int gdn_gate_quant_launch(unsigned grid, const void* o, int Tp, const void* z, int64_t ld, int z_off, const void* gw,
                          float eps, int rows, int ntok, int Hv, void* y, uint8_t* q, float* s, cudaStream_t st) {
  return launch_pdl(hybrid::gdn_gate_quant_kernel<T, TO>, grid, 256, 0, st, static_cast<const TO*>(o), Tp,
                    static_cast<const T*>(z), ld, z_off, static_cast<const T*>(gw), eps, rows, ntok, Hv,
                    static_cast<T*>(y), q, s);
}

int gdn_gate_quant(const void* o, int o_dtype, int Tp, const void* z, int dt, int64_t ld, int z_off, const void* gw,
                   float eps, int rows, int T, int Hv, void* y, uint8_t* q, float* s, cudaStream_t st) {
  if (rows < 0 || T < 0 || Hv <= 0 || Tp < T || !(eps >= 0.0f)) return BASAL200_ERR_ARG;
  if (dt != BASAL200_BF16 && dt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (o_dtype != BASAL200_F32 && o_dtype != dt) return BASAL200_ERR_DTYPE;
  if (rows == 0 || T == 0) return BASAL200_OK;
  if (!o || !z || !gw || !q || !s) return BASAL200_ERR_ARG;
  if (z_off < 0 || z_off + (int64_t)Hv * 128 > ld || (ld % 8) || (z_off % 8)) return BASAL200_ERR_SHAPE;
  if (!aligned16(o) || !aligned16(z) || !aligned16(gw) || !aligned16(q) || (y && !aligned16(y)) ||
      (reinterpret_cast<uintptr_t>(s) & 3))
    return BASAL200_ERR_ALIGN;
  const int64_t warps = ((int64_t)rows * T * Hv + 1) / 2;  // a half-warp per (token, head)
  if ((warps + 7) / 8 > INT32_MAX) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  using bf16 = __nv_bfloat16;
  const bool f32 = o_dtype == BASAL200_F32;
  if (dt == BASAL200_BF16)
    return f32 ? gdn_gate_quant_launch<bf16, float>(grid, o, Tp, z, ld, z_off, gw, eps, rows, T, Hv, y, q, s, st)
               : gdn_gate_quant_launch<bf16, bf16>(grid, o, Tp, z, ld, z_off, gw, eps, rows, T, Hv, y, q, s, st);
  return f32 ? gdn_gate_quant_launch<__half, float>(grid, o, Tp, z, ld, z_off, gw, eps, rows, T, Hv, y, q, s, st)
             : gdn_gate_quant_launch<__half, __half>(grid, o, Tp, z, ld, z_off, gw, eps, rows, T, Hv, y, q, s, st);
}

// The attention layer's input steps (q / k norms, rotary embedding, keys and values into their buffers) and its
// output gate fused with the output projection's quantiser; heads of 128.
int attn_prep(const void* qkv, int dt, int64_t ld, int rows, int T, int H, int Hk, const void* q_norm,
              const void* k_norm, float eps, const void* cos, const void* sin, int64_t cs_row, int rot, void* q_out,
              void* k_out, void* v_out, int64_t kv_len, int64_t kv_off, cudaStream_t st) {
  if (rows < 0 || T < 0 || H <= 0 || Hk <= 0 || !(eps >= 0.0f) || cs_row < 0 || kv_off < 0) return BASAL200_ERR_ARG;
  if (dt != BASAL200_BF16 && dt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (rot < 0 || rot > 128 || rot % 8 || kv_off + T > kv_len || ld < (int64_t)H * 256 + (int64_t)Hk * 256)
    return BASAL200_ERR_SHAPE;
  if (rows == 0 || T == 0) return BASAL200_OK;
  if (!qkv || !q_norm || !k_norm || !q_out || !k_out || !v_out || (rot > 0 && (!cos || !sin))) return BASAL200_ERR_ARG;
  if ((ld % 4) || (reinterpret_cast<uintptr_t>(qkv) & 7) || (reinterpret_cast<uintptr_t>(q_norm) & 7) ||
      (reinterpret_cast<uintptr_t>(k_norm) & 7) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out))
    return BASAL200_ERR_ALIGN;
  const int64_t items = (int64_t)rows * T * (H + Hk);  // a warp each, 8 a CTA
  if ((items + 7) / 8 > INT32_MAX) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  hybrid::AttnPrepParams p;
  p.qkv = qkv;
  p.ld = ld;
  p.rows = rows;
  p.T = T;
  p.H = H;
  p.Hk = Hk;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.eps = eps;
  p.cos = cos;
  p.sin = sin;
  p.cs_row = cs_row;
  p.rot = rot;
  p.q_out = q_out;
  p.k_out = k_out;
  p.v_out = v_out;
  p.kv_len = kv_len;
  p.kv_off = kv_off;
  const unsigned grid = (unsigned)((items + 7) / 8);
  if (dt == BASAL200_BF16) return launch_pdl(hybrid::attn_prep_kernel<__nv_bfloat16>, grid, 256, 0, st, p);
  return launch_pdl(hybrid::attn_prep_kernel<__half>, grid, 256, 0, st, p);
}

int attn_gate_quant(const void* o, int dt, const void* qkv, int64_t ld, int rows, int T, int H, uint8_t* q, float* s,
                    cudaStream_t st) {
  if (rows < 0 || T < 0 || H <= 0) return BASAL200_ERR_ARG;
  if (dt != BASAL200_BF16 && dt != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (ld < (int64_t)H * 256) return BASAL200_ERR_SHAPE;
  if (rows == 0 || T == 0) return BASAL200_OK;
  if (!o || !qkv || !q || !s) return BASAL200_ERR_ARG;
  if ((ld % 8) || !aligned16(o) || !aligned16(qkv) || !aligned16(q) || (reinterpret_cast<uintptr_t>(s) & 3))
    return BASAL200_ERR_ALIGN;
  const int64_t warps = ((int64_t)rows * T * H + 1) / 2;  // a half-warp per (token, head)
  if ((warps + 7) / 8 > INT32_MAX) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (dt == BASAL200_BF16)
    return launch_pdl(hybrid::attn_gate_quant_kernel<__nv_bfloat16>, grid, 256, 0, st,
                      static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(qkv), ld, rows, T, H, q,
                      s);
  return launch_pdl(hybrid::attn_gate_quant_kernel<__half>, grid, 256, 0, st, static_cast<const __half*>(o),
                    static_cast<const __half*>(qkv), ld, rows, T, H, q, s);
}

template <typename TV, typename TO>
int gdn_chunk_launch(int dev, int slot, const gdnchunk::Params& p, cudaStream_t st) {
  constexpr size_t smem = sizeof(gdnchunk::Smem);
  int rc = set_smem(dev, slot, gdnchunk::gdn_chunk_kernel<TV, TO>, smem);
  if (rc) return rc;
  return launch_pdl(gdnchunk::gdn_chunk_kernel<TV, TO>, (unsigned)(p.rows * p.H), gdnchunk::NT, smem, st, p);
}

int gdn_chunk(const float* q, const float* k, const void* v, int v_dtype, const float* g, const float* beta,
              const float* s0, int s0_rows, void* o, int o_dtype, float* s_out, int rows, int Hk, int H, int T,
              cudaStream_t st) {
  if (rows < 0 || Hk <= 0 || H <= 0 || T < 0) return BASAL200_ERR_ARG;
  if (H % Hk) return BASAL200_ERR_SHAPE;
  if (v_dtype != BASAL200_F32 && v_dtype != BASAL200_BF16 && v_dtype != BASAL200_F16) return BASAL200_ERR_DTYPE;
  if (o_dtype != BASAL200_F32 && o_dtype != v_dtype) return BASAL200_ERR_DTYPE;  // fp32, or v's 16-bit type
  if (rows == 0) return BASAL200_OK;
  if (T > 0 && (!q || !k || !v || !g || !beta || !o)) return BASAL200_ERR_ARG;  // no tokens: nothing of them is read
  if (s0 && s0_rows != 1 && s0_rows != rows) return BASAL200_ERR_ARG;
  if ((T > 0 && (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))) || (s0 && !aligned16(s0)) ||
      (s_out && !aligned16(s_out)))
    return BASAL200_ERR_ALIGN;
  if ((int64_t)rows * H > INT32_MAX || (int64_t)rows * H * T * 128 > ((int64_t)1 << 40)) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  if (T == 0) {  // no tokens: the state passes through unchanged
    if (!s_out) return BASAL200_OK;
    if (!s0) return cudaMemsetAsync(s_out, 0, (size_t)rows * H * 128 * 128 * 4, st) == cudaSuccess
                        ? BASAL200_OK : BASAL200_ERR_LAUNCH;
    for (int r = 0; r < rows; ++r)
      if (cudaMemcpyAsync(s_out + (int64_t)r * H * 128 * 128, s0 + (int64_t)(s0_rows == 1 ? 0 : r) * H * 128 * 128,
                          (size_t)H * 128 * 128 * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return BASAL200_ERR_LAUNCH;
    return BASAL200_OK;
  }
  gdnchunk::Params p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.s0 = s0;
  p.s0_rows = s0_rows;
  p.o = o;
  p.s_out = s_out;
  p.rows = rows;
  p.Hk = Hk;
  p.H = H;
  p.T = T;
  const bool f32 = o_dtype == BASAL200_F32;
  if (v_dtype == BASAL200_F32) return gdn_chunk_launch<float, float>(dev, kSlotGdn, p, st);
  if (v_dtype == BASAL200_BF16)
    return f32 ? gdn_chunk_launch<__nv_bfloat16, float>(dev, kSlotGdnV, p, st)
               : gdn_chunk_launch<__nv_bfloat16, __nv_bfloat16>(dev, kSlotGdnVO, p, st);
  return f32 ? gdn_chunk_launch<__half, float>(dev, kSlotGdnV + 1, p, st)
             : gdn_chunk_launch<__half, __half>(dev, kSlotGdnVO + 1, p, st);
}

// ------------------------------------------------------------------------------------------------------------
// Allocation-free FP8-block linear: the activation codes and scales live in one file-scope device array instead of
// caller scratch. The array is part of the loaded module, so every GPU that loads the library holds its
// 16.5 MiB until the process exits; all calls on a device share it.
// ------------------------------------------------------------------------------------------------------------
constexpr int64_t kNoAllocMaxElems = BASAL200_NOALLOC_MAX_ELEMS;              // M * K activation values at most
constexpr size_t kNoAllocCodeBytes = (size_t)kNoAllocMaxElems;                // e4m3 codes, one byte each
constexpr size_t kNoAllocScaleBytes = (size_t)(kNoAllocMaxElems / 128) * 4;  // one fp32 scale per 128 values
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocCodeBytes + kNoAllocScaleBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_base[kMaxDevices];  // the array's device address, per device ordinal (null: not set up yet)

// Host code may not take the array's address itself (on the host the symbol is only a stand-in): the runtime
// translates it, once per device, with that device current.
int noalloc_scratch(int dev, uint8_t** q, float** s) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return BASAL200_ERR_LAUNCH;
    }
    g_noalloc_base[dev] = p;
  }
  *q = static_cast<uint8_t*>(g_noalloc_base[dev]);
  *s = reinterpret_cast<float*>(static_cast<uint8_t*>(g_noalloc_base[dev]) + kNoAllocCodeBytes);
  return BASAL200_OK;
}
}  // namespace
}  // namespace b200

using namespace b200;

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int basal200_fp8_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, uint8_t* q, float* s, void* stream) {
  return act_quant<false>(x, x_dtype, M, K, q, s, as_stream(stream));
}

int basal200_int8_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* q, float* s, void* stream) {
  return act_quant<true>(x, x_dtype, M, K, q, s, as_stream(stream));
}

int basal200_fp8_block_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* q, float* s,
                                void* stream) {
  return weight_quant<false>(w, w_dtype, N, K, q, s, as_stream(stream));
}

int basal200_int8_block_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int8_t* q, float* s,
                                 void* stream) {
  return weight_quant<true>(w, w_dtype, N, K, q, s, as_stream(stream));
}

int64_t basal200_block_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) { return split_workspace(M, N, K); }

int basal200_fp8_block_gemm(const uint8_t* q, const float* s, const uint8_t* w, const float* ws, const void* bias,
                            void* c, int c_dtype, int64_t M, int64_t N, int64_t K, void* workspace,
                            int64_t workspace_bytes, void* stream) {
  return block_gemm<false>(q, s, w, ws, bias, c, c_dtype, M, N, K, workspace, workspace_bytes, as_stream(stream));
}

int basal200_fp8_block_gemm_gather(const uint8_t* q, const float* s, const uint8_t* w, const float* ws,
                                   void* const* outs, int npeers, int64_t col_off, int64_t n_total, int c_dtype,
                                   int64_t M, int64_t N, int64_t K, const uint32_t* barrier_pad, void* stream) {
  return block_gemm_gather(q, s, w, ws, outs, npeers, col_off, n_total, c_dtype, M, N, K, barrier_pad,
                           as_stream(stream));
}

int basal200_peer_barrier(uint32_t* const* pads, int world, int rank, int64_t timeout_ns, void* stream) {
  if (!pads || world < 1 || world > blockgemm::kMaxPeers || rank < 0 || rank >= world || timeout_ns <= 0)
    return BASAL200_ERR_ARG;
  blockgemm::PeerPads pp;
  for (int r = 0; r < blockgemm::kMaxPeers; ++r) {
    pp.p[r] = r < world ? pads[r] : nullptr;
    if (r < world && (!pads[r] || (reinterpret_cast<uintptr_t>(pads[r]) & 3))) return BASAL200_ERR_ALIGN;
  }
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  blockgemm::peer_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(pp, world, rank, (long long)timeout_ns);
  return launched();
}

int basal200_int8_block_gemm(const int8_t* q, const float* s, const int8_t* w, const float* ws, const void* bias,
                             void* c, int c_dtype, int64_t M, int64_t N, int64_t K, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  return block_gemm<true>(q, s, w, ws, bias, c, c_dtype, M, N, K, workspace, workspace_bytes, as_stream(stream));
}

int basal200_fp8_block_linear(const void* x, int x_dtype, const uint8_t* w, const float* ws, const void* bias,
                              void* y, int64_t M, int64_t N, int64_t K, uint8_t* q_scratch, float* s_scratch,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  if (M > 0 && (N % 128)) return BASAL200_ERR_SHAPE;
  int rc = fused_split_linear<false>(x, x_dtype, w, ws, bias, y, M, N, K, s_scratch, workspace, workspace_bytes,
                                      as_stream(stream));
  if (rc >= 0) return rc;
  rc = act_quant<false>(x, x_dtype, M, K, q_scratch, s_scratch, as_stream(stream));
  if (rc) return rc;
  return block_gemm<false>(q_scratch, s_scratch, w, ws, bias, y, x_dtype, M, N, K, workspace, workspace_bytes,
                           as_stream(stream));
}

int basal200_int8_block_linear(const void* x, int x_dtype, const int8_t* w, const float* ws, const void* bias,
                               void* y, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  if (M > 0 && (N % 128)) return BASAL200_ERR_SHAPE;
  int rc = fused_split_linear<true>(x, x_dtype, w, ws, bias, y, M, N, K, s_scratch, workspace, workspace_bytes,
                                      as_stream(stream));
  if (rc >= 0) return rc;
  rc = act_quant<true>(x, x_dtype, M, K, q_scratch, s_scratch, as_stream(stream));
  if (rc) return rc;
  return block_gemm<true>(q_scratch, s_scratch, w, ws, bias, y, x_dtype, M, N, K, workspace, workspace_bytes,
                          as_stream(stream));
}

int64_t basal200_block_linear_glu_workspace_bytes(int64_t M, int64_t I, int64_t K) { return glu_workspace(M, I, K); }

int64_t basal200_block_linear_residual_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return res_workspace(M, N, K);
}

int basal200_fp8_block_linear_residual(const void* x, int x_dtype, const uint8_t* w, const float* ws,
                                       const void* bias, const void* residual, void* y, int64_t M, int64_t N,
                                       int64_t K, uint8_t* q_scratch, float* s_scratch, void* workspace,
                                       int64_t workspace_bytes, void* stream) {
  return block_linear_residual<false>(x, x_dtype, w, ws, bias, residual, y, M, N, K, q_scratch, s_scratch, workspace,
                                      workspace_bytes, as_stream(stream));
}

int basal200_int8_block_linear_residual(const void* x, int x_dtype, const int8_t* w, const float* ws,
                                        const void* bias, const void* residual, void* y, int64_t M, int64_t N,
                                        int64_t K, int8_t* q_scratch, float* s_scratch, void* workspace,
                                        int64_t workspace_bytes, void* stream) {
  return block_linear_residual<true>(x, x_dtype, w, ws, bias, residual, y, M, N, K, q_scratch, s_scratch, workspace,
                                     workspace_bytes, as_stream(stream));
}

int basal200_fp8_block_linear_glu(const void* x, int x_dtype, const uint8_t* w, const float* ws, void* y, int64_t M,
                                  int64_t I, int64_t K, int act, uint8_t* q_scratch, float* s_scratch, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  return block_linear_glu<false>(x, x_dtype, w, ws, y, M, I, K, act, q_scratch, s_scratch, workspace,
                                 workspace_bytes, as_stream(stream));
}

int basal200_int8_block_linear_glu(const void* x, int x_dtype, const int8_t* w, const float* ws, void* y, int64_t M,
                                   int64_t I, int64_t K, int act, int8_t* q_scratch, float* s_scratch,
                                   void* workspace, int64_t workspace_bytes, void* stream) {
  return block_linear_glu<true>(x, x_dtype, w, ws, y, M, I, K, act, q_scratch, s_scratch, workspace,
                                workspace_bytes, as_stream(stream));
}

int basal200_fp8_block_gemm_glu(const uint8_t* q, const float* s, const uint8_t* w, const float* ws, void* y,
                                int y_dtype, int64_t M, int64_t I, int64_t K, int act, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  return block_linear_glu<false>(nullptr, y_dtype, w, ws, y, M, I, K, act, const_cast<uint8_t*>(q),
                                 const_cast<float*>(s), workspace, workspace_bytes, as_stream(stream), true);
}

int basal200_fp8_block_gemm_residual(const uint8_t* q, const float* s, const uint8_t* w, const float* ws,
                                     const void* bias, const void* residual, void* y, int y_dtype, int64_t M,
                                     int64_t N, int64_t K, void* workspace, int64_t workspace_bytes, void* stream) {
  return block_linear_residual<false>(nullptr, y_dtype, w, ws, bias, residual, y, M, N, K, const_cast<uint8_t*>(q),
                                      const_cast<float*>(s), workspace, workspace_bytes, as_stream(stream), true);
}

int basal200_rms_norm_fp8_quant(const void* x, int x_dtype, const void* w, float eps, int64_t M, int64_t D, void* y,
                                uint8_t* q, float* s, void* stream) {
  return rms_quant(x, x_dtype, w, eps, M, D, y, q, s, as_stream(stream));
}

int basal200_gdn_prep(const void* proj, int dtype, int64_t ld, const void* tail, int tail_rows, const void* conv,
                      int kw, const float* A_log, const void* dt_bias, int b_off, int a_off, int rows, int T, int Hk,
                      int Hv, float* q, float* k, void* v, float* beta, float* g, void* stream) {
  return gdn_prep(proj, dtype, ld, tail, tail_rows, conv, kw, A_log, dt_bias, b_off, a_off, rows, T, Hk, Hv, q, k, v,
                  beta, g, as_stream(stream));
}

int basal200_gdn_gate_fp8_quant(const void* o, int o_dtype, int Tp, const void* z, int dtype, int64_t ld, int z_off,
                                const void* gw, float eps, int rows, int T, int Hv, void* y, uint8_t* q, float* s,
                                void* stream) {
  return gdn_gate_quant(o, o_dtype, Tp, z, dtype, ld, z_off, gw, eps, rows, T, Hv, y, q, s, as_stream(stream));
}

int basal200_attn_prep(const void* qkv, int dtype, int64_t ld, int rows, int T, int H, int Hk, const void* q_norm,
                       const void* k_norm, float eps, const void* cos, const void* sin, int64_t cs_row, int rot,
                       void* q_out, void* k_out, void* v_out, int64_t kv_len, int64_t kv_off, void* stream) {
  return attn_prep(qkv, dtype, ld, rows, T, H, Hk, q_norm, k_norm, eps, cos, sin, cs_row, rot, q_out, k_out, v_out,
                   kv_len, kv_off, as_stream(stream));
}

int basal200_attn_gate_fp8_quant(const void* o, int dtype, const void* qkv, int64_t ld, int rows, int T, int H,
                                 uint8_t* q, float* s, void* stream) {
  return attn_gate_quant(o, dtype, qkv, ld, rows, T, H, q, s, as_stream(stream));
}

int basal200_gdn_chunk_rule(const float* q, const float* k, const void* v, int v_dtype, const float* g,
                            const float* beta, const float* s0, int s0_rows, void* o, int o_dtype, float* s_out,
                            int rows, int Hk, int H, int T, void* stream) {
  return gdn_chunk(q, k, v, v_dtype, g, beta, s0, s0_rows, o, o_dtype, s_out, rows, Hk, H, T, as_stream(stream));
}

// The two kernels of basal200_fp8_block_linear, the quantiser writing into the library's own device array. Nothing
// there needs clearing between calls: the quantiser writes every code and scale the GEMM then reads, and rows past M
// are zero-filled by the GEMM's TMA loads, never read from the array.
int basal200_fp8_block_linear_noalloc(const void* x, int x_dtype, const uint8_t* w, const float* ws,
                                      const void* bias, void* y, int64_t M, int64_t N, int64_t K, void* stream) {
  if (M < 0 || K <= 0) return BASAL200_ERR_ARG;
  if (M > 0 && (N % 128)) return BASAL200_ERR_SHAPE;
  if (M > kNoAllocMaxElems / K) return BASAL200_ERR_LIMIT;
  if (M == 0) return BASAL200_OK;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  uint8_t* q = nullptr;
  float* s = nullptr;
  if ((rc = noalloc_scratch(dev, &q, &s))) return rc;
  rc = act_quant<false>(x, x_dtype, M, K, q, s, as_stream(stream));
  if (rc) return rc;
  return block_gemm<false>(q, s, w, ws, bias, y, x_dtype, M, N, K, nullptr, 0, as_stream(stream));
}

int basal200_nvfp4_act_quant(const void* x, int x_dtype, const float* inv_g, int64_t M, int64_t K, uint8_t* q,
                             uint8_t* s, void* stream) {
  return nvfp4_act(x, x_dtype, inv_g, M, K, q, s, as_stream(stream));
}

int basal200_nvfp4_gemm(const uint8_t* q, const uint8_t* s, const uint8_t* w, const uint8_t* ws, const float* alpha,
                        const void* bias, void* y, int y_dtype, int64_t M, int64_t N, int64_t K, void* stream) {
  return fp4_gemm(q, s, w, ws, alpha, bias, y, y_dtype, M, N, K, as_stream(stream));
}

int basal200_nvfp4_linear(const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws, const float* alpha,
                          const float* inv_g, const void* bias, void* y, int64_t M, int64_t N, int64_t K,
                          uint8_t* q_scratch, uint8_t* s_scratch, void* stream) {
  if (M > 0 && (N % 16)) return BASAL200_ERR_SHAPE;
  int rc = nvfp4_act(x, x_dtype, inv_g, M, K, q_scratch, s_scratch, as_stream(stream));
  if (rc) return rc;
  return fp4_gemm(q_scratch, s_scratch, w, ws, alpha, bias, y, x_dtype, M, N, K, as_stream(stream));
}

int basal200_nvfp4_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* codes, uint8_t* scales,
                            float* g, void* stream) {
  if (N <= 0 || K <= 0 || !w || !codes || !scales || !g) return BASAL200_ERR_ARG;
  if (K % 16) return BASAL200_ERR_SHAPE;
  if (!aligned16(w) || !aligned16(codes)) return BASAL200_ERR_ALIGN;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  switch (w_dtype) {
    case BASAL200_BF16:
      return nvfp4_wq_typed(static_cast<const __nv_bfloat16*>(w), N, K, codes, scales, g, dev, st);
    case BASAL200_F16: return nvfp4_wq_typed(static_cast<const __half*>(w), N, K, codes, scales, g, dev, st);
    case BASAL200_F32: return nvfp4_wq_typed(static_cast<const float*>(w), N, K, codes, scales, g, dev, st);
    default: return BASAL200_ERR_DTYPE;
  }
}

int basal200_code_logits(const void* h, int h_dtype, int64_t R, int64_t D, int64_t ldh, const void* head,
                         int head_dtype, int64_t V, int64_t ldw, const int64_t* ids, int64_t U, const void* bias,
                         int bias_dtype, float softcap, float* z, void* stream) {
  if (R < 0 || U < 0 || V <= 0 || D <= 0 || ldh < D || ldw < D) return BASAL200_ERR_ARG;
  if (R == 0 || U == 0) return BASAL200_OK;
  if (!h || !head || !ids || !z) return BASAL200_ERR_ARG;
  if (R > INT32_MAX || U > INT32_MAX) return BASAL200_ERR_LIMIT;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  switch (h_dtype) {
    case BASAL200_BF16:
      return logits_head(dev, static_cast<const __nv_bfloat16*>(h), R, D, ldh, head, head_dtype, V, ldw, ids, U, bias,
                         bias_dtype, softcap, z, st);
    case BASAL200_F16:
      return logits_head(dev, static_cast<const __half*>(h), R, D, ldh, head, head_dtype, V, ldw, ids, U, bias,
                         bias_dtype, softcap, z, st);
    case BASAL200_F32:
      return logits_head(dev, static_cast<const float*>(h), R, D, ldh, head, head_dtype, V, ldw, ids, U, bias,
                         bias_dtype, softcap, z, st);
    default:
      return BASAL200_ERR_DTYPE;
  }
}

int basal200_code_probs(const float* z, int64_t R, int64_t U, const int64_t* idx, const uint8_t* pad, int64_t Kmax,
                        float* p, void* stream) {
  if (R < 0 || U < 0 || Kmax < 0) return BASAL200_ERR_ARG;
  if (Kmax > 1024) return BASAL200_ERR_LIMIT;
  if (R == 0 || Kmax == 0) return BASAL200_OK;
  if (!z || !idx || !p) return BASAL200_ERR_ARG;
  int dev, rc = current_device(&dev);
  if (rc) return rc;
  const unsigned grid = (unsigned)((R + 7) / 8);
  cudaStream_t st = as_stream(stream);
  if (Kmax <= 32) return launch_pdl(readout::code_probs_kernel<1>, grid, 256, 0, st, z, R, U, idx, pad, Kmax, p);
  if (Kmax <= 64) return launch_pdl(readout::code_probs_kernel<2>, grid, 256, 0, st, z, R, U, idx, pad, Kmax, p);
  if (Kmax <= 128) return launch_pdl(readout::code_probs_kernel<4>, grid, 256, 0, st, z, R, U, idx, pad, Kmax, p);
  if (Kmax <= 256) return launch_pdl(readout::code_probs_kernel<8>, grid, 256, 0, st, z, R, U, idx, pad, Kmax, p);
  return launch_pdl(readout::code_probs_kernel<32>, grid, 256, 0, st, z, R, U, idx, pad, Kmax, p);
}

unsigned basal200_device_faults(int device, int clear) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  unsigned v = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_fault, sizeof(v));
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_fault, &zero, sizeof(zero));
  }
  cudaSetDevice(prev);
  return v;
}

const char* basal200_status_string(int status) {
  switch (status) {
    case BASAL200_OK: return "ok";
    case BASAL200_ERR_ARG: return "invalid argument (null pointer or negative size)";
    case BASAL200_ERR_SHAPE: return "shape not supported by the format";
    case BASAL200_ERR_ALIGN: return "pointer not 16-byte aligned";
    case BASAL200_ERR_DTYPE: return "unsupported dtype";
    case BASAL200_ERR_ARCH: return "the current device is not sm_100 (B200)";
    case BASAL200_ERR_LAUNCH: return "CUDA launch error";
    case BASAL200_ERR_TMAP: return "TMA descriptor could not be encoded";
    case BASAL200_ERR_LIMIT: return "size beyond the supported limit";
    default: return "unknown status";
  }
}

int basal200_version(void) { return 1; }

}  // extern "C"
