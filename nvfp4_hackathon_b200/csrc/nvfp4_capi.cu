// C-ABI of the NVFP4 B200 library (declared in include/nvfp4_b200.h).
//
// Host responsibilities: argument checks, TMA tensor-map encoding (through the
// driver entry point, so the library does not link libcuda), tile-shape
// dispatch, and the launch on the caller's stream.  Nothing here synchronises
// the stream; device-side errors (timed-out waits) land in a status word that
// nvfp4_status_get() reads.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "nvfp4_kernels.cuh"
#include "nvfp4_quant.cuh"
#include "../../include/nvfp4_b200.h"

using namespace nvfp4;

// ------------------------------------------------------------------ status word
// One word per device that loads the library; kernels record the first error here.
__device__ int g_nvfp4_status;

namespace {

constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // 2 s per wait

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(NVFP4_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

struct DeviceState {
  bool init = false;
  int num_sms = 0;
  int* status = nullptr;  // device address of g_nvfp4_status
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::atomic<unsigned long long> g_timeout_ns{kDefaultTimeoutNs};

int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    e = cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(NVFP4_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only",
                  dev, major, minor);
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.status), g_nvfp4_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(NVFP4_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not available");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    st.init = true;
  }
  *out = &st;
  return NVFP4_OK;
}

// Operand map: a (rows x kbytes x batch) uint8 tensor, K-major, box = box_inner bytes of
// K (128 -> 128-byte swizzle, 64 -> 64-byte swizzle) x box_rows rows.  Out-of-range rows
// read as zero.
int encode_operand_map(CUtensorMap* m, const void* ptr, long long rows, long long kbytes,
                       long long batch, int box_rows, int box_inner = 128) {
  cuuint64_t dims[3] = {(cuuint64_t)kbytes, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)kbytes, (cuuint64_t)(rows * kbytes)};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        box_inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d) rows=%lld kbytes=%lld", (int)r,
                rows, kbytes);
  return NVFP4_OK;
}

// Scale-factor map of one operand's permuted scales (L, ceil(mn/128), K/64 atoms of 512
// bytes) seen as 8-byte elements: row = one 128-row block, box = the KB atoms of one
// k-stage of `blocks` consecutive blocks.  Out-of-range blocks and atoms read as zero.
int encode_sf_map(CUtensorMap* m, const void* ptr, long long mn, long long k, long long batch,
                  int kb, int blocks) {
  const long long rk = (k + 63) / 64, rest = (mn + 127) / 128;
  cuuint64_t dims[3] = {(cuuint64_t)(rk * 64), (cuuint64_t)rest, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(rk * kAtomBytes), (cuuint64_t)(rest * rk * kAtomBytes)};
  cuuint32_t box[3] = {(cuuint32_t)(kb * 64), (cuuint32_t)blocks, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_INT64, 3, const_cast<void*>(ptr), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_DRIVER, "cuTensorMapEncodeTiled (scales) failed (%d) mn=%lld k=%lld",
                (int)r, mn, k);
  return NVFP4_OK;
}

// Store map of C (fp16 / bf16, (L, M, N) row-major, row stride N) for the TMA epilogue: the
// box is 16 columns x 32 rows (32-byte rows, 32-byte swizzle), or for the swapped operand
// order 32 columns x 16 rows (64-byte rows, 64-byte swizzle).  Needs N % 8 == 0 and a
// 16-byte aligned C (TMA strides and base).
int encode_c_map(CUtensorMap* m, const void* ptr, long long rows, long long cols, long long batch,
                 bool swap) {
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(cols * 2), (cuuint64_t)(rows * cols * 2)};
  cuuint32_t box[3] = {swap ? 32u : 16u, swap ? 16u : 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(ptr), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swap ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_DRIVER, "cuTensorMapEncodeTiled (C) failed (%d) rows=%lld cols=%lld", (int)r,
                rows, cols);
  return NVFP4_OK;
}

// Per-thread memo of recent operand maps: a repeated call on the same buffers skips
// the driver encode (about a microsecond each).  The key covers every input of the
// encoding, so a hit is exactly the map the driver would build again.
struct MapKey {
  const void* ptr;
  long long rows, kbytes, batch;
  int box_rows, box_inner;
  int kind;  // 0 operand map, 1 scale-factor map, 2 C store map
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && kbytes == o.kbytes && batch == o.batch &&
           box_rows == o.box_rows && box_inner == o.box_inner && kind == o.kind;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCache = 16;
thread_local MapEntry g_map_cache[kMapCache];
thread_local int g_map_next = 0;

int cached_map(CUtensorMap* m, int kind, const void* ptr, long long rows, long long kbytes,
               long long batch, int box_rows, int box_inner) {
  const MapKey key{ptr, rows, kbytes, batch, box_rows, box_inner, kind};
  for (int i = 0; i < kMapCache; ++i)
    if (g_map_cache[i].valid && g_map_cache[i].key == key) {
      *m = g_map_cache[i].map;
      return NVFP4_OK;
    }
  // (scale maps: rows = mn, kbytes = k, box_rows = blocks, box_inner = KB;
  //  C maps: rows = m, kbytes = n, box_inner = operand order swapped)
  int rc = kind == 0   ? encode_operand_map(m, ptr, rows, kbytes, batch, box_rows, box_inner)
           : kind == 1 ? encode_sf_map(m, ptr, rows, kbytes, batch, box_inner, box_rows)
                       : encode_c_map(m, ptr, rows, kbytes, batch, box_inner != 0);
  if (rc) return rc;
  MapEntry& e = g_map_cache[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.key = key;
  e.map = *m;
  e.valid = true;
  return NVFP4_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with programmatic stream serialization: the kernel may start while the
// previous kernel on the stream finishes; it calls griddepcontrol.wait before it
// touches global memory.  `coop`: cooperative launch (all CTAs co-resident), for grids
// whose CTAs wait on one another.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       int cluster, bool coop, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (coop) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e;
}

template <bool GROUPED, bool SWAP, int BN, int KB, bool CTA2 = false, bool SK = false, bool F32 = false>
int launch(const CUtensorMap& tp, const CUtensorMap& tq, const CUtensorMap& tsp,
           const CUtensorMap& tsq, const CUtensorMap& tc, const GemmParams& prm, int grid,
           cudaStream_t stream) {
  using C_ = Cfg<BN, KB, CTA2>;
  auto kern = nvfp4_gemm_kernel<GROUPED, SWAP, BN, KB, CTA2, SK, F32>;
  // the shared-memory opt-in is per device and per kernel; concurrent host threads may
  // race to set it, which is harmless (same value), but the flag itself is atomic
  static std::atomic<bool> attr_done[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = C_::kSmemBytes;
  if (!attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    attr_done[dev].store(true, std::memory_order_release);
  }
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kNumThreads), smem, stream,
                             CTA2 ? 2 : 1, SK, tp, tq, tsp, tsq, tc, prm);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_gemm_kernel launch");
  return NVFP4_OK;
}

struct DenseChoice {
  bool swap;
  int bn;
  int kb;    // 64-wide K blocks per stage (2 or 4)
  bool cta2; // M = 256 tiles over a CTA pair (tcgen05 cta_group::2)
};

DenseChoice choose_dense(int m, int n, int k, const nvfp4_options* opt) {
  (void)k;
  DenseChoice c;
  // M >= 256 with a wide N: M = 256 x N = 256 tiles on a CTA pair (each SM stages 128 rows of
  // A and 128 of B per k-step instead of 128 + 256: a third fewer bytes per MMA cycle).
  if (m <= 64) c = {true, 64, 4, false};
  else if (m <= 128) c = {true, 128, 4, false};
  else if (m >= 256 && n >= 2048 && !(opt && opt->out_dtype == 2)) c = {false, 256, 4, true};
  else c = {false, (n >= 2048) ? 256 : 128, 4, false};
  if (opt) {
    if (opt->cta_pair == 1) c.cta2 = false;
    if (opt->cta_pair == 2) c.cta2 = true;
    if (opt->stage_k == 128) c.kb = 2;
    if (opt->stage_k == 256) c.kb = 4;
    if (opt->operand_order == 1) c.swap = false;
    if (opt->operand_order == 2) c.swap = true;
    if (opt->tile_n > 0) c.bn = opt->tile_n;
  }
  return c;
}

// Stream-K workspace of one (device, stream): a flag per CTA (up to kSkMaxCtas) and one
// fp32 partial tile (128 x BN) per CTA in kSkSlotsBytes.  Allocated on first use and kept.
// On a stream that is being captured into a graph, the one-time allocation is made outside
// the capture (relaxed capture mode for this thread), and the graph keeps using it.  The
// flags are cleared by a memset on the stream before every stream-K launch.
constexpr int kSkMaxCtas = 1024;
constexpr size_t kSkSlotsBytes = 16u << 20;
struct SkWorkspace {
  int dev;
  cudaStream_t stream;
  void* ptr;
};
std::mutex g_sk_mu;
std::vector<SkWorkspace> g_sk;

void* sk_workspace(int dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_sk_mu);
  for (const SkWorkspace& w : g_sk)
    if (w.dev == dev && w.stream == stream) return w.ptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  void* p = nullptr;
  const size_t bytes = kSkMaxCtas * sizeof(unsigned) + kSkSlotsBytes;
  if (cap == cudaStreamCaptureStatusNone) {
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
  } else {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t e = cudaMalloc(&p, bytes);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
  }
  g_sk.push_back({dev, stream, p});
  return p;
}

// Several destinations for one dense GEMM's C (nvfp4_gemm_multi): set for the duration of
// that call on this thread only.
struct MultiOut {
  int n;
  long long ldc;
  const void* ptr[8];
};
thread_local const MultiOut* g_multi_out = nullptr;

template <bool SWAP, int BN, int KB, bool CTA2 = false>
int run_dense_bn(const void* a, const void* b, const void* sfa, const void* sfb, void* c, int m,
                 int n, int k, int l, cudaStream_t stream, DeviceState* st,
                 const nvfp4_options* opt) {
  // P feeds the 128-row MMA side, Q the BN side.
  const void* P = SWAP ? b : a;
  const void* Q = SWAP ? a : b;
  const void* sfP = SWAP ? sfb : sfa;
  const void* sfQ = SWAP ? sfa : sfb;
  const int p_rows = SWAP ? n : m;
  const int q_rows = SWAP ? m : n;
  const long long kbytes = k / 2;
  CUtensorMap tp, tq, tsp, tsq;
  int rc = cached_map(&tp, 0, P, p_rows, kbytes, l, kBM, KB * 32);
  if (rc) return rc;
  rc = cached_map(&tq, 0, Q, q_rows, kbytes, l, CTA2 ? BN / 2 : BN, KB * 32);
  if (rc) return rc;
  rc = cached_map(&tsp, 1, sfP, p_rows, k, l, 1, KB);
  if (rc) return rc;
  rc = cached_map(&tsq, 1, sfQ, q_rows, k, l, Cfg<BN, KB, CTA2>::kSfqAtoms, KB);
  if (rc) return rc;
  // TMA-store epilogue: one fp16/bf16 output buffer with 16-byte rows strides
  const bool c_tma = !g_multi_out && !(opt && opt->out_dtype == 2) && n % 8 == 0 && aligned16(c);
  CUtensorMap tc = tp;  // (unused unless c_tma)
  if (c_tma) {
    rc = cached_map(&tc, 2, c, m, n, l, 0, SWAP ? 1 : 0);
    if (rc) return rc;
  }
  GemmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.p_rows = p_rows;
  prm.q_rows = q_rows;
  prm.K = k;
  prm.L = l;
  prm.C = static_cast<__half*>(c);
  prm.ldc = n;
  if (g_multi_out) {
    prm.n_out = g_multi_out->n;
    prm.ldc = g_multi_out->ldc;
    for (int i = 0; i < g_multi_out->n; ++i)
      prm.outs[i] = reinterpret_cast<unsigned long long>(g_multi_out->ptr[i]);
  }
  prm.c_batch = (long long)m * n;
  const int pm = CTA2 ? 2 * kBM : kBM;  // P rows per tile (a CTA pair covers 256)
  prm.tiles_p = (p_rows + pm - 1) / pm;
  prm.tiles_q = (q_rows + BN - 1) / BN;
  const long long total = (long long)prm.tiles_p * prm.tiles_q * l;
  if (total > 0x7fffffffLL) return fail(NVFP4_ERR_UNSUPPORTED, "too many tiles");
  prm.total_tiles = (int)total;
  // Raster bands of P tiles whose operand rows (over all of K) total about 32 MB, so a band's
  // P rows stay in L2 while the Q tiles stream past them (16384 x 28672 x 8192 read 2.9 GB
  // from DRAM with P fastest over all 64 P tiles, against 0.21 GB of operands).
  {
    const long long band_bytes = (long long)pm * (k / 2 + k / 16);
    long long bp = (32ll << 20) / (band_bytes > 0 ? band_bytes : 1);
    if (bp < 1) bp = 1;
    if (bp > prm.tiles_p) bp = prm.tiles_p;
    prm.band_p = (int)bp;
  }
  prm.c_tma = c_tma ? 1 : 0;
  prm.status = (opt && opt->dev_status) ? opt->dev_status : st->status;
  prm.timeout_ns = (opt && opt->timeout_ns) ? opt->timeout_ns : g_timeout_ns.load();
  prm.debug = opt ? (opt->debug & 1) : 0;
  if (opt) {
    prm.bias = opt->bias;
    prm.act = opt->activation;
    prm.out_bf16 = opt->out_dtype == 1;
  }
  int grid = st->num_sms;
  if (opt && opt->max_ctas > 0 && opt->max_ctas < grid) grid = opt->max_ctas;
  if (CTA2) {
    int pairs = grid / 2;
    if (pairs > prm.total_tiles) pairs = prm.total_tiles;
    if (pairs < 1) pairs = 1;
    grid = 2 * pairs;
  } else if (grid > prm.total_tiles) {
    grid = prm.total_tiles;
  }
  // Stream-K (option stream_k = 2; off by default): every CTA takes an equal share of all
  // k-steps and a split tile's fp32 partials meet in the CTA holding its k-step 0.  Measured
  // on B200 against the plain schedule it does not pay for these skinny shapes (M = 128:
  // 128 x 4096 x 7168 20.5 vs 15.3 us, 128 x 1536 x 7168 18.7 vs 14.8 us, 128 x 7168 x 16384
  // 30.2 vs 30.4 us; c1 15.6 vs 12.2 us): the HBM stream of the tiles' CTAs is already close
  // to what more SMs get, and the reduction adds an L2 round trip.  BN <= 128, no CTA pairs.
  const int ktn = (k + KB * 64 - 1) / (KB * 64);
  const int sk_opt = opt ? opt->stream_k : 0;
  const bool sk_auto = false;
  if constexpr (!CTA2 && BN <= 128) if (ktn >= 2 && (sk_opt == 2 || sk_auto)) {
    int g = st->num_sms;
    if (opt && opt->max_ctas > 0 && opt->max_ctas < g) g = opt->max_ctas;
    if ((long long)prm.total_tiles * ktn < g) g = prm.total_tiles * ktn;
    int dev = 0;
    cudaGetDevice(&dev);
    void* ws = (g <= kSkMaxCtas && (size_t)g * BN * 128 * sizeof(float) <= kSkSlotsBytes &&
                (long long)prm.total_tiles * ktn < 0x7fffffffLL)
                   ? sk_workspace(dev, stream) : nullptr;
    // every flag starts clear, whatever an earlier launch (even one that timed out) left
    if (ws && g > prm.total_tiles &&
        cudaMemsetAsync(ws, 0, (size_t)g * sizeof(unsigned), stream) == cudaSuccess) {
      prm.sk_ktn = ktn;
      prm.sk_flags = static_cast<unsigned*>(ws);
      prm.sk_slots = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kSkMaxCtas * sizeof(unsigned));
      rc = launch<false, SWAP, BN, KB, CTA2, true>(tp, tq, tsp, tsq, tc, prm, g, stream);
      if (rc == NVFP4_OK) return rc;
      // (a cooperative launch the device refuses: run the plain schedule instead)
      cudaGetLastError();
      prm.sk_ktn = 0;
    }
  }
  if (opt && opt->out_dtype == 2) {
    if constexpr (CTA2) return fail(NVFP4_ERR_UNSUPPORTED, "fp32 C is not built for CTA pairs");
    else return launch<false, SWAP, BN, KB, false, false, true>(tp, tq, tsp, tsq, tc, prm, grid, stream);
  }
  return launch<false, SWAP, BN, KB, CTA2>(tp, tq, tsp, tsq, tc, prm, grid, stream);
}

// ------------------------------------------------------------------ grouped GEMM
constexpr int kMaxGroups = 1024;
// token rows per tile (MMA N side): fewer token tiles per group means fewer re-reads of
// the group's B_g, which outweighs the MMA width lost on small groups (G=64 Zipf experts:
// 305 us at 256 against 392 us at 128)
constexpr int kGroupedBN = 256;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t grouped_ws_bytes(int G) {
  return align_up((size_t)G * 5 * sizeof(CUtensorMap), 256) + align_up((size_t)(G + 1) * 4, 256);
}

__device__ __forceinline__ void tmap_replace_addr(void* m, const void* p) {
  asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "l"(reinterpret_cast<uint64_t>(p))
               : "memory");
}
template <int ORD>
__device__ __forceinline__ void tmap_replace_dim(void* m, uint32_t v) {
  asm volatile("tensormap.replace.tile.global_dim.global.b1024.b32 [%0], %1, %2;" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "n"(ORD), "r"(v)
               : "memory");
}
template <int ORD>
__device__ __forceinline__ void tmap_replace_stride(void* m, uint64_t v) {
  asm volatile("tensormap.replace.tile.global_stride.global.b1024.b64 [%0], %1, %2;" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "n"(ORD), "l"(v)
               : "memory");
}

// One thread per group: validate the group, clone the three template maps into
// the workspace and point them at the group's B (P side), A (Q side) and C (the TMA
// store map, when n % 8 == 0 and C is 16-byte aligned), then a block-wide scan turns
// per-group tile counts into the schedule prefix.
__global__ void __launch_bounds__(kMaxGroups)
nvfp4_grouped_prep(const __grid_constant__ CUtensorMap tmpl_p, const __grid_constant__ CUtensorMap tmpl_q,
                   const __grid_constant__ CUtensorMap tmpl_c, const __grid_constant__ CUtensorMap tmpl_sfp,
                   const __grid_constant__ CUtensorMap tmpl_sfq, const int* __restrict__ sizes,
                   const unsigned long long* __restrict__ abc,
                   const unsigned long long* __restrict__ sfs, int G, CUtensorMap* maps,
                   int* prefix, int pm, int bn, int swap, int* status) {
  __shared__ int warp_sums[kMaxGroups / 32];
  pdl_launch_dependents();
  // the workspace may still be read by the previous call's GEMM on this stream
  pdl_wait_prior_grid();
  const int g = threadIdx.x;
  int tiles = 0;
  if (g < G) {
    const int m = sizes[4 * g + 0], n = sizes[4 * g + 1], k = sizes[4 * g + 2], l = sizes[4 * g + 3];
    const unsigned long long pa = abc[3 * g + 0], pb = abc[3 * g + 1], pc = abc[3 * g + 2];
    const unsigned long long sa = sfs[2 * g + 0], sb = sfs[2 * g + 1];
    const bool empty = (m == 0 || n == 0);
    const bool valid = m >= 0 && n >= 0 && l == 1 && k >= 64 && (k % 64) == 0 &&
                       ((pa | pb | sa | sb) & 15ull) == 0 && (pc & 1ull) == 0 &&
                       (empty || (pa && pb && pc && sa && sb));
    if (!valid) {
      atomicCAS(status, 0, 5 /* NVFP4_STATUS_BAD_GROUP */);
    } else if (!empty) {
      // (pm = 256 for CTA pairs; swapped: B_g rows on the pm side, tokens on the bn side)
      tiles = swap ? ((n + pm - 1) / pm) * ((m + bn - 1) / bn) : ((m + pm - 1) / pm) * ((n + bn - 1) / bn);
      CUtensorMap* mp = maps + 5 * g;
      CUtensorMap* mq = maps + 5 * g + 1;
      *mp = tmpl_p;
      *mq = tmpl_q;
      const uint64_t kbytes = (uint64_t)k / 2;
      const unsigned long long p_ptr = swap ? pb : pa, q_ptr = swap ? pa : pb;
      const uint32_t p_rows = (uint32_t)(swap ? n : m), q_rows = (uint32_t)(swap ? m : n);
      tmap_replace_addr(mp, reinterpret_cast<const void*>(p_ptr));
      tmap_replace_dim<0>(mp, (uint32_t)kbytes);
      tmap_replace_dim<1>(mp, p_rows);
      tmap_replace_stride<0>(mp, kbytes);
      tmap_replace_stride<1>(mp, kbytes * (uint64_t)p_rows);
      tmap_replace_addr(mq, reinterpret_cast<const void*>(q_ptr));
      tmap_replace_dim<0>(mq, (uint32_t)kbytes);
      tmap_replace_dim<1>(mq, q_rows);
      tmap_replace_stride<0>(mq, kbytes);
      tmap_replace_stride<1>(mq, kbytes * (uint64_t)q_rows);
      // scale maps: permuted scales as 8-byte elements, row = one 128-row block
      {
        const uint64_t rk = (uint64_t)k / 64;
        const unsigned long long sp = swap ? sb : sa, sq = swap ? sa : sb;
        const uint32_t bp = (p_rows + 127) / 128, bq = (q_rows + 127) / 128;
        CUtensorMap* ms = maps + 5 * g + 3;
        CUtensorMap* mt = maps + 5 * g + 4;
        *ms = tmpl_sfp;
        *mt = tmpl_sfq;
        tmap_replace_addr(ms, reinterpret_cast<const void*>(sp));
        tmap_replace_dim<0>(ms, (uint32_t)(rk * 64));
        tmap_replace_dim<1>(ms, bp);
        tmap_replace_stride<0>(ms, rk * kAtomBytes);
        tmap_replace_stride<1>(ms, rk * kAtomBytes * bp);
        tmap_replace_addr(mt, reinterpret_cast<const void*>(sq));
        tmap_replace_dim<0>(mt, (uint32_t)(rk * 64));
        tmap_replace_dim<1>(mt, bq);
        tmap_replace_stride<0>(mt, rk * kAtomBytes);
        tmap_replace_stride<1>(mt, rk * kAtomBytes * bq);
      }
      if ((n & 7) == 0 && (pc & 15ull) == 0) {
        CUtensorMap* mc = maps + 5 * g + 2;
        *mc = tmpl_c;
        tmap_replace_addr(mc, reinterpret_cast<const void*>(pc));
        tmap_replace_dim<0>(mc, (uint32_t)n);
        tmap_replace_dim<1>(mc, (uint32_t)m);
        tmap_replace_stride<0>(mc, 2ull * (uint64_t)n);
        tmap_replace_stride<1>(mc, 2ull * (uint64_t)n * (uint64_t)m);
      }
      asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
    }
  }
  // inclusive block scan of tile counts
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int v = tiles;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_sums[wid] = v;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x / 32;
    int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    if (lane < nw) warp_sums[lane] = w;
  }
  __syncthreads();
  const int incl = v + (wid > 0 ? warp_sums[wid - 1] : 0);
  if (g < G) prefix[g + 1] = incl;
  if (g == 0) prefix[0] = 0;
}

template <int BN, int KB = 4, bool CTA2 = false, bool SWAP = true>
int run_grouped_bn(const int32_t* sizes, const uint64_t* abc, const uint64_t* sfs, int G, void* ws,
                   cudaStream_t stream, DeviceState* st, const nvfp4_options* opt) {
  // Templates: any valid 16-byte-aligned address and sizes; the prep kernel
  // replaces address, extents and strides per group.
  CUtensorMap tp, tq;
  int rc = encode_operand_map(&tp, ws, 128, 128, 1, kBM, KB * 32);
  if (rc) return rc;
  rc = encode_operand_map(&tq, ws, 128, 128, 1, CTA2 ? BN / 2 : BN, KB * 32);
  if (rc) return rc;
  CUtensorMap tc;
  rc = encode_c_map(&tc, ws, 64, 64, 1, SWAP);
  if (rc) return rc;
  CUtensorMap tsp, tsq;  // scale-map templates: the box (one k-stage of 1 or 2 blocks) is kept
  rc = encode_sf_map(&tsp, ws, 128, 256, 1, KB, 1);
  if (rc) return rc;
  rc = encode_sf_map(&tsq, ws, 256, 256, 1, KB, Cfg<BN, KB, CTA2>::kSfqAtoms);
  if (rc) return rc;
  CUtensorMap* maps = static_cast<CUtensorMap*>(ws);
  int* prefix = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) +
                                       align_up((size_t)G * 5 * sizeof(CUtensorMap), 256));
  const int threads = ((G + 31) / 32) * 32;
  cudaError_t e = launch_pdl(nvfp4_grouped_prep, dim3(1), dim3(threads), 0, stream, 1, false, tp, tq, tc, tsp, tsq, sizes,
                             reinterpret_cast<const unsigned long long*>(abc),
                             reinterpret_cast<const unsigned long long*>(sfs), G, maps, prefix,
                             CTA2 ? 2 * kBM : kBM, BN, SWAP ? 1 : 0,
                             (opt && opt->dev_status) ? opt->dev_status : st->status);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_grouped_prep launch");
  GemmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.G = G;
  prm.sizes = sizes;
  prm.abc = reinterpret_cast<const unsigned long long*>(abc);
  prm.sfs = reinterpret_cast<const unsigned long long*>(sfs);
  prm.maps = maps;
  prm.tile_prefix = prefix;
  prm.status = (opt && opt->dev_status) ? opt->dev_status : st->status;
  prm.timeout_ns = (opt && opt->timeout_ns) ? opt->timeout_ns : g_timeout_ns.load();
  prm.debug = opt ? (opt->debug & 1) : 0;
  int grid = st->num_sms;
  if (opt && opt->max_ctas > 0 && opt->max_ctas < grid) grid = opt->max_ctas;
  if (CTA2) grid = grid / 2 < 1 ? 2 : grid / 2 * 2;  // whole pairs
  // (the grouped kernel's operand, scale and C maps are the per-group ones in the workspace)
  return launch<true, SWAP, BN, KB, CTA2>(tp, tq, tsp, tsq, tc, prm, grid, stream);
}

}  // namespace

// ======================================================================= C ABI
extern "C" {

const char* nvfp4_last_error(void) { return g_last_error.c_str(); }

int nvfp4_abi_version(void) { return NVFP4_ABI_VERSION; }

int nvfp4_set_timeout_ns(unsigned long long ns) {
  g_timeout_ns = ns ? ns : kDefaultTimeoutNs;
  return NVFP4_OK;
}

int nvfp4_status_get(int* out) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_nvfp4_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (out) *out = v;
  return NVFP4_OK;
}

int nvfp4_status_reset(void) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_nvfp4_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  return NVFP4_OK;
}

int nvfp4_gemm_ex(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm, void* c,
                  int m, int n, int k, int l, void* stream, const nvfp4_options* opt) {
  if (!a || !b || !sfa_perm || !sfb_perm || !c)
    return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if (m <= 0 || n <= 0 || k <= 0 || l <= 0)
    return fail(NVFP4_ERR_INVALID_ARG, "m, n, k, l must be positive (got %d, %d, %d, %d)", m, n, k, l);
  if (k % 64 != 0)
    return fail(NVFP4_ERR_UNSUPPORTED, "k must be a multiple of 64 (got %d)", k);
  if (!aligned16(a) || !aligned16(b) || !aligned16(sfa_perm) || !aligned16(sfb_perm))
    return fail(NVFP4_ERR_ALIGNMENT, "a, b and the scale tensors must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(c) & 1u) != 0)
    return fail(NVFP4_ERR_ALIGNMENT, "c must be 2-byte aligned");
  if (opt && (opt->activation < 0 || opt->activation > 2 || opt->out_dtype < 0 || opt->out_dtype > 2))
    return fail(NVFP4_ERR_INVALID_ARG, "activation must be 0..2 and out_dtype 0..2");
  if (opt && opt->out_dtype == 2 && (reinterpret_cast<uintptr_t>(c) & 3u) != 0)
    return fail(NVFP4_ERR_ALIGNMENT, "an fp32 c must be 4-byte aligned");
  if (opt && opt->out_dtype == 2 && opt->stream_k == 2)
    return fail(NVFP4_ERR_UNSUPPORTED, "stream-K stores fp16 or bf16 only");
  if (opt && opt->bias && (reinterpret_cast<uintptr_t>(opt->bias) & 3u) != 0)
    return fail(NVFP4_ERR_ALIGNMENT, "bias must be 4-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DenseChoice ch = choose_dense(m, n, k, opt);
#define NVFP4_DENSE_CASE(SW, BNV, KBV)                                                    \
  if (!ch.cta2 && ch.swap == SW && ch.bn == BNV && ch.kb == KBV)                                      \
    return run_dense_bn<SW, BNV, KBV>(a, b, sfa_perm, sfb_perm, c, m, n, k, l, s, st, opt);
  NVFP4_DENSE_CASE(true, 64, 4)
  NVFP4_DENSE_CASE(true, 128, 4)
  NVFP4_DENSE_CASE(true, 256, 4)
  NVFP4_DENSE_CASE(false, 64, 4)
  NVFP4_DENSE_CASE(false, 128, 4)
  NVFP4_DENSE_CASE(false, 256, 4)
  NVFP4_DENSE_CASE(true, 64, 2)
  NVFP4_DENSE_CASE(true, 128, 2)
  NVFP4_DENSE_CASE(false, 128, 2)
  NVFP4_DENSE_CASE(false, 256, 2)
#undef NVFP4_DENSE_CASE
#define NVFP4_PAIR_CASE(SW, BNV)                                                              \
  if (ch.cta2 && ch.swap == SW && ch.bn == BNV && ch.kb == 4)                                   \
    return run_dense_bn<SW, BNV, 4, true>(a, b, sfa_perm, sfb_perm, c, m, n, k, l, s, st, opt);
  NVFP4_PAIR_CASE(true, 64)
  NVFP4_PAIR_CASE(true, 128)
  NVFP4_PAIR_CASE(false, 128)
  NVFP4_PAIR_CASE(false, 256)
#undef NVFP4_PAIR_CASE
#undef NVFP4_DENSE_CASE
  return fail(NVFP4_ERR_UNSUPPORTED, "no kernel for swap=%d tile_n=%d stage_k=%d", (int)ch.swap, ch.bn,
              ch.kb * 64);
}

int nvfp4_gemm_multi(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm,
                     const void* const* outs, int n_out, long long ldc, int m, int n, int k,
                     void* stream) {
  if (!outs || n_out < 1 || n_out > 8)
    return fail(NVFP4_ERR_INVALID_ARG, "1..8 output buffers (got %d)", n_out);
  if (ldc < n) return fail(NVFP4_ERR_INVALID_ARG, "ldc %lld < n %d", ldc, n);
  MultiOut mo;
  mo.n = n_out;
  mo.ldc = ldc;
  for (int i = 0; i < n_out; ++i) {
    if (!outs[i] || (reinterpret_cast<uintptr_t>(outs[i]) & 1u))
      return fail(NVFP4_ERR_ALIGNMENT, "output %d null or not 2-byte aligned", i);
    mo.ptr[i] = outs[i];
  }
  g_multi_out = &mo;
  const int rc = nvfp4_gemm_ex(a, b, sfa_perm, sfb_perm, const_cast<void*>(outs[0]), m, n, k, 1,
                               stream, nullptr);
  g_multi_out = nullptr;
  return rc;
}

int nvfp4_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int nvfp4_ipc_get_handle(const void* dev_ptr, void* handle_out, unsigned long long* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return fail(NVFP4_ERR_INVALID_ARG, "null pointer");
  // the handle names the whole allocation holding dev_ptr; its opener adds the offset back
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return fail(NVFP4_ERR_DRIVER, "cuMemGetAddressRange not available");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(NVFP4_ERR_DRIVER, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (unsigned long long)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return NVFP4_OK;
}

int nvfp4_ipc_open_handle(const void* handle, void** dev_ptr_out) {
  // (returns the base of the exporter's allocation: add the exporter's offset)
  if (!handle || !dev_ptr_out) return fail(NVFP4_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return NVFP4_OK;
}

int nvfp4_ipc_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return NVFP4_OK;
}

int nvfp4_gemm(const void* a, const void* b, const void* sfa_perm, const void* sfb_perm, void* c,
               int m, int n, int k, int l, void* stream) {
  return nvfp4_gemm_ex(a, b, sfa_perm, sfb_perm, c, m, n, k, l, stream, nullptr);
}

size_t nvfp4_grouped_gemm_workspace_size(int G) {
  if (G <= 0 || G > kMaxGroups) return 0;
  return grouped_ws_bytes(G);
}

int nvfp4_grouped_gemm_ex(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                          const uint64_t* sf_ptrs_dev, int G, void* workspace,
                          size_t workspace_bytes, void* stream, const nvfp4_options* opt) {
  if (opt && (opt->bias || opt->activation || opt->out_dtype))
    return fail(NVFP4_ERR_UNSUPPORTED, "the fused epilogue (bias, activation, out_dtype) is dense-only");
  if (G <= 0 || G > kMaxGroups)
    return fail(NVFP4_ERR_UNSUPPORTED, "group count %d outside [1, %d]", G, kMaxGroups);
  if (!sizes_dev || !abc_ptrs_dev || !sf_ptrs_dev)
    return fail(NVFP4_ERR_INVALID_ARG, "null group table");
  if (!workspace || workspace_bytes < grouped_ws_bytes(G))
    return fail(NVFP4_ERR_WORKSPACE, "workspace needs %zu bytes", grouped_ws_bytes(G));
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NVFP4_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bn = (opt && opt->tile_n > 0) ? opt->tile_n : kGroupedBN;
  if (opt && opt->operand_order == 1) {
    // A_g (tokens) on the 128-row MMA side, B_g rows on the N side: tiles of 128 tokens x bn
    // rows of B_g (or 256 tokens on a CTA pair); fewer MMA instructions than the swapped
    // order when groups hold many tokens, since only the last 128-token tile is padded
    if (opt->cta_pair == 2 && bn == 256)
      return run_grouped_bn<256, 4, true, false>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    if (opt->cta_pair != 2 && bn == 256 && opt->stage_k == 128)
      return run_grouped_bn<256, 2, false, false>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    if (opt->cta_pair != 2 && bn == 256)
      return run_grouped_bn<256, 4, false, false>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    if (opt->cta_pair != 2 && bn == 128)
      return run_grouped_bn<128, 4, false, false>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    return fail(NVFP4_ERR_UNSUPPORTED, "grouped operand_order 1 is built for tile_n 128, 256 (pair: 256)");
  }
  if (opt && opt->cta_pair == 2) {  // 256 rows of B_g per tile on a CTA pair
    if (bn == 128) return run_grouped_bn<128, 4, true>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    if (bn == 256) return run_grouped_bn<256, 4, true>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    return fail(NVFP4_ERR_UNSUPPORTED, "grouped CTA pairs are built for tile_n 128 and 256 (got %d)", bn);
  }
  switch (bn) {
    case 64: return run_grouped_bn<64>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    case 128:
      if (opt && opt->stage_k == 128)
        return run_grouped_bn<128, 2>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
      return run_grouped_bn<128>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    case 192: return run_grouped_bn<192>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    case 256: return run_grouped_bn<256>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, s, st, opt);
    default: return fail(NVFP4_ERR_UNSUPPORTED, "grouped tile_n %d not built", bn);
  }
}

int nvfp4_grouped_gemm(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                       const uint64_t* sf_ptrs_dev, int G, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return nvfp4_grouped_gemm_ex(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, workspace, workspace_bytes,
                               stream, nullptr);
}

int nvfp4_quantize(const void* x, int dtype, int rows, int k, int l, void* codes, void* sf_perm,
                   void* sf_plain, void* stream) {
  if (!x || !codes || !sf_perm) return fail(NVFP4_ERR_INVALID_ARG, "null pointer");
  if (rows <= 0 || l <= 0 || k <= 0) return fail(NVFP4_ERR_INVALID_ARG, "non-positive size");
  if (k % 64) return fail(NVFP4_ERR_UNSUPPORTED, "k must be a multiple of 64 (got %d)", k);
  if (dtype < kQuantF32 || dtype > kQuantBF16) return fail(NVFP4_ERR_INVALID_ARG, "dtype %d", dtype);
  if (!aligned16(x) || !aligned16(codes) || !aligned16(sf_perm))
    return fail(NVFP4_ERR_ALIGNMENT, "x, codes and sf_perm must be 16-byte aligned");
  const int rm = (rows + 127) / 128;
  if (rm > 65535 || l > 65535) return fail(NVFP4_ERR_UNSUPPORTED, "too many rows or batches");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const int atoms = dtype == kQuantF32 ? quant_atoms<kQuantF32>() : quant_atoms<kQuantF16>();
  const dim3 grid((k / 64 + atoms - 1) / atoms, rm, l);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* c8 = static_cast<uint8_t*>(codes);
  auto* sp = static_cast<uint8_t*>(sf_perm);
  auto* pl = static_cast<uint8_t*>(sf_plain);
  if (dtype == kQuantF32) nvfp4_quantize_kernel<kQuantF32><<<grid, 256, 0, s>>>(x, rows, k, c8, sp, pl);
  else if (dtype == kQuantF16) nvfp4_quantize_kernel<kQuantF16><<<grid, 256, 0, s>>>(x, rows, k, c8, sp, pl);
  else nvfp4_quantize_kernel<kQuantBF16><<<grid, 256, 0, s>>>(x, rows, k, c8, sp, pl);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_quantize_kernel launch");
  return NVFP4_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ grouped GEMM without allocation
// Scratch for nvfp4_grouped_gemm_noalloc: room for the per-group tensor maps and
// the tile prefix of up to kNoAllocMaxGroups groups (about 161 KiB).  Every GPU
// that loads the library holds one copy until the process exits.  In host code
// the name below is only a host-side stand-in; the device address comes from
// cudaGetSymbolAddress, once per device.
constexpr int kNoAllocMaxGroups = 256;
constexpr size_t kNoAllocScratchBytes =
    ((size_t)kNoAllocMaxGroups * 5 * sizeof(CUtensorMap) + 255) / 256 * 256 +
    ((size_t)(kNoAllocMaxGroups + 1) * 4 + 255) / 256 * 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

extern "C" int nvfp4_grouped_gemm_noalloc(const int32_t* sizes_dev, const uint64_t* abc_ptrs_dev,
                                          const uint64_t* sf_ptrs_dev, int G, void* stream) {
  if (G <= 0 || G > kNoAllocMaxGroups)
    return fail(NVFP4_ERR_UNSUPPORTED,
                "nvfp4_grouped_gemm_noalloc handles 1..%d groups (got %d); use nvfp4_grouped_gemm "
                "with a caller-allocated workspace for more",
                kNoAllocMaxGroups, G);
  if (!sizes_dev || !abc_ptrs_dev || !sf_ptrs_dev)
    return fail(NVFP4_ERR_INVALID_ARG, "null group table");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      // first call on this device (the current one): look up the array's device address
      e = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_ptr[dev] = nullptr;
        return cuda_fail(e, "cudaGetSymbolAddress(grouped scratch)");
      }
    }
    scratch = g_noalloc_ptr[dev];
  }
  if (grouped_ws_bytes(G) > kNoAllocScratchBytes)
    return fail(NVFP4_ERR_WORKSPACE, "internal: scratch too small for %d groups", G);
  // The prep kernel rewrites the tile prefix and the maps of every non-empty
  // group on each call, so nothing in the scratch has to start at zero.
  return run_grouped_bn<kGroupedBN>(sizes_dev, abc_ptrs_dev, sf_ptrs_dev, G, scratch,
                                    static_cast<cudaStream_t>(stream), st, nullptr);
}
