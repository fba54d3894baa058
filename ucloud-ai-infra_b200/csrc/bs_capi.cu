// C-ABI entry points of libbs_fp8_sm100.so: argument checks, TMA descriptor creation, kernel
// selection and launch. One translation unit so that every kernel can name the status word.
#include <algorithm>
#include <mutex>
#include <utility>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <cudaTypedefs.h>

#include "bs_common.cuh"
#include "bs_prefill.cuh"
#include "bs_decode.cuh"
#include "bs_quant.cuh"
#include "bs_tp.cuh"
#include "../../include/bs_fp8.h"

// Library status word: kernels record the first bounded-wait timeout here.
__device__ int g_bs_status;

namespace {

constexpr int kMaxDevices = 64;

// Text of the last CUDA runtime failure seen by this library on the calling thread.
thread_local char g_last_cuda_error[256] = "";

int cuda_fail(cudaError_t e, const char* where) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s (%s)", where, cudaGetErrorName(e),
                cudaGetErrorString(e));
  return BS_ERR_CUDA;
}

// Launch result: the launch's own error, not an older one left in the runtime's error slot.
int launch_status(const char* where) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BS_OK : cuda_fail(e, where);
}

struct DeviceState {
  std::once_flag once;
  int num_sms = 0;
  int* status = nullptr;
  int err = 0;
};
DeviceState g_dev[kMaxDevices];

std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// Per-device set-up (SM count, status word address), done once per device with that device current.
DeviceState* device_state() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  DeviceState* d = &g_dev[dev];
  std::call_once(d->once, [d, dev] {
    cudaError_t e = cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) d->err = cuda_fail(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
    // BS_FP8_SM_LIMIT caps the CTAs of the persistent GEMM kernels, leaving the other SMs to kernels
    // that run at the same time (e.g. the collectives of a tensor-parallel layer).
    if (const char* v = std::getenv("BS_FP8_SM_LIMIT")) {
      const long lim = std::strtol(v, nullptr, 10);
      if (lim >= 8 && lim < d->num_sms) d->num_sms = static_cast<int>(lim);
    }
    void* sym = nullptr;
    e = cudaGetSymbolAddress(&sym, g_bs_status);
    if (e != cudaSuccess) d->err = cuda_fail(e, "cudaGetSymbolAddress(status word)");
    d->status = static_cast<int*>(sym);
  });
  return d->err ? nullptr : d;
}

// 2-D uint8 tensor map with a 128-byte-swizzled box (operand loads) or a plain box (stores of
// row-major tiles); out-of-range elements read as zero and are never written.
int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
             uint32_t box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = encoder();
  if (!enc) return BS_ERR_TMAP;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BS_OK : BS_ERR_TMAP;
}

// Weight map: tile-first [N*K/128 rows of 128 bytes] or row-major [N rows of K bytes], with boxes of
// `box_rows` weight rows x 128 bytes (128: whole weight blocks; 64: the fused prefill's half blocks).
int make_weight_map(CUtensorMap* m, const void* B, int N, int K, int tiled, int box_rows = 128) {
  if (tiled)
    return make_map(m, B, 128, static_cast<uint64_t>(N) * (K / 128), 128, 128, box_rows);
  return make_map(m, B, K, N, K, 128, box_rows);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ntp_for(int M) { return ((M + 15) / 16) * 16; }

// Prefill row count from which 256-row tiles on CTA pairs (cta_group::2) are used. Measured on B200
// (K = 5120): the fused gate_up kernel is faster on pairs from M = 1024 (8192 rows: 1891 vs 1826
// TFLOP/s), where each CTA stages 32 KB per K block instead of 48 KB; the plain GEMM is slower on pairs
// (1716 vs 1938), so it stays on one CTA per tile. BS_FP8_PAIR_MIN_ROWS, read once per process,
// replaces both thresholds (a very large value turns pairs off).
int pair_min_rows(bool fused) {
  struct Rows {
    int fused = 1024;
    int plain = 0x7fffffff;
  };
  static std::once_flag once;
  static Rows rows;
  std::call_once(once, [] {
    const char* v = std::getenv("BS_FP8_PAIR_MIN_ROWS");
    if (v && *v) {
      const long r = std::strtol(v, nullptr, 10);
      if (r > 0 && r <= 0x7fffffff) rows.fused = rows.plain = static_cast<int>(r);
    }
  });
  return fused ? rows.fused : rows.plain;
}

// Grid of the decode kernels. When the weight tiles nearly match the SM count (>= 90%), one CTA
// per tile streams whole tiles and no tile is split (no partial sums, no finishing CTA). When a
// whole number s of CTAs per tile still fills >= 95% of the SMs, each tile is split into s equal
// K ranges (every CTA holds one segment of one tile: one fix-up, none at a tile boundary).
// Otherwise the stream-K split over one CTA per SM keeps every SM streaming equal bytes. Never
// more CTAs than (tile, K block) units.
// *split (optional) receives the choice: 0 one CTA per tile, s > 0 equal K splits, -1 stream-K.
int decode_grid(int num_sms, int tiles, int KB, int* split = nullptr) {
  int sp = -1, grid;
  if (tiles <= num_sms && 10 * tiles >= 9 * num_sms) {
    sp = 0;
    grid = tiles;
  } else if (tiles < num_sms && num_sms / tiles >= 2 && num_sms / tiles <= KB &&
             20 * tiles * (num_sms / tiles) >= 19 * num_sms) {
    sp = num_sms / tiles;
    grid = tiles * sp;
  } else {
    const long long units = static_cast<long long>(tiles) * KB;
    grid = static_cast<int>(units < num_sms ? units : num_sms);
  }
  if (split) *split = sp;
  return grid;
}

// Decode workspace layout: a fixed prefix of kCounterBytes holds one arrival counter per weight tile (up to
// kMaxDecodeTiles tiles), then the fp32 partial tiles of the split-K CTAs. The prefix does not depend on the
// shape and the kernels leave every counter they use at zero, so one zero-filled workspace serves any sequence
// of shapes (a layout sized by the tile count would put the counters of a wider call where a narrower call
// left partial sums).
constexpr int kMaxDecodeTiles = 16384;
constexpr size_t kCounterBytes = static_cast<size_t>(kMaxDecodeTiles) * 4;

size_t decode_ws_bytes(int G, int nwg, int ntp) {
  return kCounterBytes + static_cast<size_t>(G) * 2 * nwg * ntp * 128 * sizeof(float);
}

// One-time per (kernel, device) preparation: opt in to the kernel's dynamic shared memory and,
// for kernels that move registers between warpgroups with setmaxnreg, check that the build gave
// them exactly the launch register count the split was computed for. The state is keyed on the
// kernel itself (a template value parameter), since all GEMM kernels share one signature.
template <auto kernel>
int prepare_kernel(int smem_bytes, int launch_regs) {
  struct State {
    std::once_flag once[kMaxDevices];
    int rc[kMaxDevices];
  };
  static State st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BS_ERR_CUDA;
  std::call_once(st.once[dev], [&] {
    int rc = BS_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
    if (rc == BS_OK && launch_regs > 0) {
      cudaFuncAttributes attr;
      e = cudaFuncGetAttributes(&attr, kernel);
      if (e != cudaSuccess)
        rc = cuda_fail(e, "cudaFuncGetAttributes");
      else if (attr.numRegs != launch_regs)
        rc = BS_ERR_BUILD;
    }
    st.rc[dev] = rc;
  });
  return st.rc[dev];
}

// Launches a library kernel as a programmatic dependent launch: it may begin while the previous
// kernel on the stream is still running, and its threads wait (griddepcontrol.wait) before any
// global access that could depend on that kernel.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kern)(KArgs...), int grid, int block, int smem, int cluster, cudaStream_t s,
                       const char* where, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  cudaGetLastError();  // clear an older error so the check below sees this launch only
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, where);
  return launch_status(where);
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), int grid, int block, int smem, cudaStream_t s, const char* where,
               Args&&... args) {
  return launch_pdl_cluster(kern, grid, block, smem, 1, s, where, std::forward<Args>(args)...);
}

template <bool FUSED, int NTP>
int launch_decode(const CUtensorMap& tmW, const CUtensorMap& tmX, const CUtensorMap& tmO, const bs::GemmParams& p,
                  int grid, cudaStream_t s) {
  using Cfg = bs::DecodeCfg<FUSED, NTP>;
  constexpr auto kern = bs::k_decode<FUSED, NTP>;
  const int rc = prepare_kernel<kern>(Cfg::kSmemBytes, Cfg::kLaunchRegs);
  if (rc != BS_OK) return rc;
  return launch_pdl(kern, grid, Cfg::kThreads, Cfg::kSmemBytes, s, "k_decode launch", tmW, tmX, tmO, p);
}

template <bool FUSED>
int dispatch_decode(int ntp, const CUtensorMap& tmW, const CUtensorMap& tmX, const CUtensorMap& tmO,
                    const bs::GemmParams& p, int grid, cudaStream_t s) {
  switch (ntp) {
    case 16: return launch_decode<FUSED, 16>(tmW, tmX, tmO, p, grid, s);
    case 32: return launch_decode<FUSED, 32>(tmW, tmX, tmO, p, grid, s);
    case 48: return launch_decode<FUSED, 48>(tmW, tmX, tmO, p, grid, s);
    case 64: return launch_decode<FUSED, 64>(tmW, tmX, tmO, p, grid, s);
    case 80: return launch_decode<FUSED, 80>(tmW, tmX, tmO, p, grid, s);
    case 96: return launch_decode<FUSED, 96>(tmW, tmX, tmO, p, grid, s);
    case 112: return launch_decode<FUSED, 112>(tmW, tmX, tmO, p, grid, s);
    case 128: return launch_decode<FUSED, 128>(tmW, tmX, tmO, p, grid, s);
    default: return BS_ERR_ARG;
  }
}

// Compile-time configuration of the decode kernel for `ntp` tokens: stages, threads, TMEM columns,
// promotion warpgroups, dynamic shared memory. False for a token count no kernel is built for.
template <bool FUSED, int NTP>
void decode_cfg_fill(int* v) {
  using C = bs::DecodeCfg<FUSED, NTP>;
  v[0] = C::kStages;
  v[1] = C::kThreads;
  v[2] = C::kTmemCols;
  v[3] = C::kPwg;
  v[4] = C::kSmemBytes;
}
template <bool FUSED>
bool decode_cfg_values(int ntp, int* v) {
  switch (ntp) {
    case 16: decode_cfg_fill<FUSED, 16>(v); return true;
    case 32: decode_cfg_fill<FUSED, 32>(v); return true;
    case 48: decode_cfg_fill<FUSED, 48>(v); return true;
    case 64: decode_cfg_fill<FUSED, 64>(v); return true;
    case 80: decode_cfg_fill<FUSED, 80>(v); return true;
    case 96: decode_cfg_fill<FUSED, 96>(v); return true;
    case 112: decode_cfg_fill<FUSED, 112>(v); return true;
    case 128: decode_cfg_fill<FUSED, 128>(v); return true;
    default: return false;
  }
}

// Clusters of two of `kern` that fit on the device at once (0 if the query fails).
template <auto kernel>
int max_pair_clusters(int threads, int smem) {
  struct State {
    std::once_flag once[kMaxDevices];
    int n[kMaxDevices];
  };
  static State st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(st.once[dev], [&] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) n = 0;
    cudaGetLastError();
    st.n[dev] = n;
  });
  return st.n[dev];
}

// Persistent prefill launch. PAIR: clusters of two CTAs on one TPC compute 256-row tiles with
// cta_group::2 MMAs, one cluster per co-resident SM pair.
template <bool FUSED, bool PAIR, bool SK = false>
int launch_prefill(const CUtensorMap& tmA, const CUtensorMap& tmB, const bs::GemmParams& p, int num_tiles,
                   int num_sms, cudaStream_t s) {
  using Cfg = bs::PrefillCfg<FUSED, PAIR>;
  constexpr auto kern = bs::k_prefill<FUSED, PAIR, SK>;
  const int rc = prepare_kernel<kern>(Cfg::kSmemBytes, Cfg::Regs::kLaunch);
  if (rc != BS_OK) return rc;
  if constexpr (PAIR) {
    int pairs = max_pair_clusters<kern>(Cfg::kThreads, Cfg::kSmemBytes);
    if (pairs <= 0) pairs = num_sms / 2;
    if (pairs > num_tiles) pairs = num_tiles;
    return launch_pdl_cluster(kern, 2 * pairs, Cfg::kThreads, Cfg::kSmemBytes, 2, s, "k_prefill<pair> launch", tmA,
                              tmB, p);
  }
  const int grid = num_tiles < num_sms ? num_tiles : num_sms;
  return launch_pdl(kern, grid, Cfg::kThreads, Cfg::kSmemBytes, s, "k_prefill launch", tmA, tmB, p);
}

// Tile walk of a prefill GEMM (M > 128): tile shape and raster.
struct PrefillPlan {
  bool pair;             // 256-row tiles on CTA pairs (cta_group::2)
  bool stream_k;         // plain, one CTA per tile: equal (tile, K block) ranges per CTA (given a workspace)
  int rows;              // output rows per tile
  int num_m, num_n;      // tiles along M and N
  int group_m;           // M tiles per raster group (see prefill_tile_coords)
};

// Stream-K workspace of the plain prefill kernel on G CTAs: the 64 KB counter prefix, then two fp32 partial
// tiles (128 rows x 256 columns) per CTA.
size_t prefill_ws_bytes(int G) { return kCounterBytes + static_cast<size_t>(G) * 2 * 128 * 256 * 4; }

PrefillPlan prefill_plan(bool fused, int M, int N, int K, int num_sms) {
  PrefillPlan pl;
  pl.pair = M >= pair_min_rows(fused);
  pl.rows = pl.pair ? 256 : 128;
  pl.num_m = (M + pl.rows - 1) / pl.rows;
  pl.num_n = fused ? N / 256 : (N / 128 + 1) / 2;
  // One group over every M tile when the whole activation panel stays in L2 (each weight tile is then read
  // from HBM once), else groups of 2048 rows. Measured on the down_proj at M = 8192 (activations 142.6 MB,
  // weights 89 MB): 0.77 GB of DRAM traffic per launch with 2048-row groups, 1.17 GB with 3584-row groups
  // (weights evict_first), 1.13 GB sweeping rows with the weights kept in L2, all at the same time (the
  // kernel is not DRAM-bound there).
  pl.group_m = static_cast<long long>(M) * K <= (48ll << 20) ? pl.num_m : 2048 / pl.rows;
  // Stream-K when whole tiles would use less than 60 % of the SM-waves they take (down_proj at M = 1024: 160
  // tiles on 148 SMs take two full tile times for 1.08 tiles of work per SM) and K is long enough (32+ blocks)
  // for the partial-tile exchange to pay. Measured: down_proj M = 1024 141 -> 109 us, o_proj M = 1024 57.5 ->
  // 50.3 us; slower: at 72-86 % of the waves (qkv at M = 1024, down_proj at M = 4096), where stream-K's CTAs
  // spread over every tile at once instead of sharing panels in L2, and at K = 1024 (19 -> 24 us).
  const long long tiles = static_cast<long long>(pl.num_m) * pl.num_n;
  const long long waves = (tiles + num_sms - 1) / num_sms;
  pl.stream_k = !fused && !pl.pair && K / 128 >= 32 && tiles > num_sms && tiles <= kMaxDecodeTiles &&
                10 * tiles < 6 * waves * num_sms;
  return pl;
}

// Argument, pointer and alignment checks shared by every GEMM entry point (BS_OK for M == 0 too; the
// callers return before launching anything then).
int validate_gemm(bool fused, const void* A, const void* B, const void* out, const float* As, const float* Bs,
                  const float* qs, int M, int N, int K, int ldc, int b_tiled, int out_dtype) {
  if (M < 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 128 != 0) return BS_ERR_ARG;
  if (fused && N % 256 != 0) return BS_ERR_ARG;
  if (!fused && (ldc < N || ldc % 8 != 0 || (out_dtype != 0 && out_dtype != 1))) return BS_ERR_ARG;
  if (b_tiled != 0 && b_tiled != 1) return BS_ERR_ARG;
  if (M == 0) return BS_OK;
  if (!A || !B || !out || !As || !Bs || (fused && !qs)) return BS_ERR_ARG;
  if (!aligned16(A) || !aligned16(B) || !aligned16(out)) return BS_ERR_ALIGN;
  return BS_OK;
}

// Shared body of bs_fp8_gemm / bs_fp8_gemm_silu_quant / bs_fp8_gemm_reduce_multicast.
int run_gemm(bool fused, const void* A, const void* B, void* out, const float* As, const float* Bs, float* qs,
             int M, int N, int K, int ldc, int b_tiled, int out_dtype, void* ws, size_t ws_bytes, void* stream,
             int out_mc = 0) {
  // (prefill: a workspace is optional; given one of bs_fp8_workspace_bytes' size, shapes whose tiles fill the
  // last wave poorly run stream-K, else every prefill shape runs whole tiles)
  const int vrc = validate_gemm(fused, A, B, out, As, Bs, qs, M, N, K, ldc, b_tiled, out_dtype);
  if (vrc != BS_OK || M == 0) return vrc;
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  bs::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.KB = K / 128;
  p.ldc = fused ? N / 2 : ldc;
  p.b_tiled = b_tiled;
  p.out_f32 = fused ? 0 : out_dtype;
  p.out_mc = out_mc;

  p.As = As;
  p.Bs = Bs;
  p.out = out;
  p.qs = qs;
  p.status = d->status;

  CUtensorMap tmB;
  if (make_weight_map(&tmB, B, N, K, b_tiled) != BS_OK) return BS_ERR_TMAP;

  if (M <= 128) {
    const int ntp = ntp_for(M);
    const int nwg = fused ? 2 : 1;
    const int tiles = fused ? N / 256 : N / 128;
    const int grid = decode_grid(d->num_sms, tiles, K / 128);
    // the kernel indexes (tile, K block) units with 32-bit products unit * grid
    if (static_cast<long long>(tiles) * (K / 128) * grid >= (1ll << 31)) return BS_ERR_ARG;
    if (tiles > kMaxDecodeTiles) return BS_ERR_ARG;
    const size_t need = decode_ws_bytes(grid, nwg, ntp);
    if (!ws || ws_bytes < need || !aligned16(ws)) return BS_ERR_WORKSPACE;
    p.cnt = static_cast<int*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes);
    CUtensorMap tmX;
    if (make_map(&tmX, A, K, M, K, 128, ntp) != BS_OK) return BS_ERR_TMAP;
    if (!fused) return dispatch_decode<false>(ntp, tmB, tmX, tmX, p, grid, s);
    // fused: the quantised output Q [M, I] is written tile by tile with TMA stores
    CUtensorMap tmO;
    if (make_map(&tmO, out, N / 2, M, N / 2, 128, ntp, CU_TENSOR_MAP_SWIZZLE_NONE) != BS_OK) return BS_ERR_TMAP;
    return dispatch_decode<true>(ntp, tmB, tmX, tmO, p, grid, s);
  }

  CUtensorMap tmA;
  if (make_map(&tmA, A, K, M, K, 128, 128) != BS_OK) return BS_ERR_TMAP;
  // the fused kernel interleaves gate and up weight rows in 64-row halves
  if (fused && make_weight_map(&tmB, B, N, K, b_tiled, 64) != BS_OK) return BS_ERR_TMAP;
  const PrefillPlan pl = prefill_plan(fused, M, N, K, d->num_sms);
  p.group_m = pl.group_m;
  const int tiles = pl.num_m * pl.num_n;
  if (pl.stream_k && !out_mc && ws && aligned16(ws) && ws_bytes >= prefill_ws_bytes(d->num_sms)) {
    p.cnt = static_cast<int*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes);
    return launch_prefill<false, false, true>(tmA, tmB, p, tiles, d->num_sms, s);
  }
  if (pl.pair)
    return fused ? launch_prefill<true, true>(tmA, tmB, p, tiles, d->num_sms, s)
                 : launch_prefill<false, true>(tmA, tmB, p, tiles, d->num_sms, s);
  return fused ? launch_prefill<true, false>(tmA, tmB, p, tiles, d->num_sms, s)
               : launch_prefill<false, false>(tmA, tmB, p, tiles, d->num_sms, s);
}

// ------------------------------------------------------------ allocation-free GEMM entry point
// Some callers cannot call cudaMalloc: an engine that reserves all device memory up front and
// forbids allocations afterwards, an embedding whose only allocator is its own arena, or a host
// thread that must never block on the driver's allocator. bs_fp8_gemm_noalloc serves them: the
// decode kernel's split-K scratch (per-tile arrival counters and fp32 partial tiles) lives in
// this fixed array, which every GPU that loads the library holds until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB: counters + partial tiles
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory, so the kernel
// gets the array's device address, looked up once per device (with that device current).
struct NoAllocScratch {
  std::once_flag once[kMaxDevices];
  void* ptr[kMaxDevices] = {};
  int rc[kMaxDevices] = {};
};
NoAllocScratch g_noalloc;

int noalloc_scratch(void** out) {
  int dev = 0;
  const cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return cuda_fail(e0, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return BS_ERR_CUDA;
  std::call_once(g_noalloc.once[dev], [dev] {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc.rc[dev] = e == cudaSuccess ? BS_OK : cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc.ptr[dev] = p;
  });
  *out = g_noalloc.ptr[dev];
  return g_noalloc.rc[dev];
}

__global__ void k_selftest_wait(uint64_t limit_ns, int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    bs::mbar_init(&bar, 1);
    abort_flag = 0;
    bs::fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must give up after limit_ns.
  if (threadIdx.x == 0) bs::mbar_wait(&bar, 0, &abort_flag, status, bs::kErrTimeoutSelftest, limit_ns);
}

}  // namespace

namespace {
using RowKernel = void (*)(const __nv_bfloat16*, int, __nv_bfloat16*, int, const __nv_bfloat16*, float, uint8_t*,
                           float*, int, int);
// k_row_group_quant for K (at most 16384): built for 1..8 chunks of 16 bytes per thread.
template <bool NORM, bool RES>
RowKernel row_kernel(int K) {
  const int c = (K / 8 + bs::kNormThreads - 1) / bs::kNormThreads;
  switch (c) {
    case 1: return bs::k_row_group_quant<1, NORM, RES>;
    case 2: return bs::k_row_group_quant<2, NORM, RES>;
    case 3: return bs::k_row_group_quant<3, NORM, RES>;
    case 4: return bs::k_row_group_quant<4, NORM, RES>;
    case 5:
    case 6: return bs::k_row_group_quant<6, NORM, RES>;
    default: return bs::k_row_group_quant<8, NORM, RES>;
  }
}
// Persistent row walk: as many CTAs as fit on the SMs at once (at most four per SM), each walking rows
// gridDim.x apart.
int launch_row_quant(RowKernel kern, int num_sms, const void* x, int ldx, void* residual, int ldr, const void* weight,
                     float eps, void* A, float* As, int M, int K, void* stream, const char* where) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, bs::kNormThreads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  cudaGetLastError();
  if (per_sm > 4) per_sm = 4;
  const int grid = M < per_sm * num_sms ? M : per_sm * num_sms;
  return launch_pdl(kern, grid, bs::kNormThreads, 0, static_cast<cudaStream_t>(stream), where,
                    static_cast<const __nv_bfloat16*>(x), ldx, static_cast<__nv_bfloat16*>(residual), ldr,
                    static_cast<const __nv_bfloat16*>(weight), eps, static_cast<uint8_t*>(A), As, M, K);
}
}  // namespace

extern "C" {

int bs_fp8_gemm(const void* A, const void* B, void* C, const float* As, const float* Bs, int M, int N, int K,
                int ldc, int b_tiled, int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return run_gemm(false, A, B, C, As, Bs, nullptr, M, N, K, ldc, b_tiled, out_dtype, workspace, workspace_bytes,
                  stream);
}

int bs_fp8_gemm_silu_quant(const void* A, const void* B, void* Q, const float* As, const float* Bs, float* Qs,
                           int M, int N2, int K, int b_tiled, void* workspace, size_t workspace_bytes,
                           void* stream) {
  return run_gemm(true, A, B, Q, As, Bs, Qs, M, N2, K, N2 / 2, b_tiled, 0, workspace, workspace_bytes, stream);
}

int bs_fp8_gemm_noalloc(const void* A, const void* B, void* C, const float* As, const float* Bs, int M, int N, int K,
                        int ldc, int b_tiled, int out_dtype, void* stream) {
  // Shapes above 128 rows run the prefill kernel, which needs no scratch; decode shapes use the
  // static array, and are refused when their scratch would not fit in it. A call that is refused
  // touches nothing: every check runs before the counters are cleared.
  const int vrc = validate_gemm(false, A, B, C, As, Bs, nullptr, M, N, K, ldc, b_tiled, out_dtype);
  if (vrc != BS_OK || M == 0) return vrc;
  if (M <= 128) {
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != BS_OK) return rc;
    DeviceState* d = device_state();
    if (!d) return BS_ERR_CUDA;
    const int tiles = N / 128;
    if (tiles > kMaxDecodeTiles) return BS_ERR_ARG;
    const size_t need = decode_ws_bytes(decode_grid(d->num_sms, tiles, K / 128), 1, ntp_for(M));
    if (need > kNoAllocScratchBytes) return BS_ERR_SCRATCH;
    // The array keeps the previous call's contents; the counters this call uses must start at zero.
    const size_t counters = static_cast<size_t>(tiles) * 4;
    const cudaError_t e = cudaMemsetAsync(scratch, 0, counters, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(no-alloc counters)");
    return run_gemm(false, A, B, C, As, Bs, nullptr, M, N, K, ldc, b_tiled, out_dtype, scratch,
                    kNoAllocScratchBytes, stream);
  }
  return run_gemm(false, A, B, C, As, Bs, nullptr, M, N, K, ldc, b_tiled, out_dtype, nullptr, 0, stream);
}

int bs_fp8_gemm_reduce_multicast(const void* A, const void* B, void* C_mc, const float* As, const float* Bs, int M,
                                 int N, int K, int ldc, int b_tiled, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  return run_gemm(false, A, B, C_mc, As, Bs, nullptr, M, N, K, ldc, b_tiled, 0, workspace, workspace_bytes, stream,
                  1);
}

long long bs_fp8_tp_flag_words(int world) {
  return world < 2 ? 0 : 2ll * bs::kTpMaxCtas * world;
}

int bs_fp8_tp_reduce_switch(unsigned long long data_mc, void* flags, unsigned long long flags_mc, long long count,
                            int rank, int world, unsigned int epoch, unsigned long long limit_ns, void* stream) {
  if (world < 2 || world > 64 || rank < 0 || rank >= world || count < 0 || count % 8) return BS_ERR_ARG;
  if (!data_mc || !flags || !flags_mc || epoch == 0) return BS_ERR_ARG;
  if (data_mc % 16 || flags_mc % 4 || !aligned16(flags)) return BS_ERR_ALIGN;
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  const long long nvec = count / 8;
  const long long per_rank = (nvec + world - 1) / world;
  // one vector per thread at least; the same on every rank (same GPU type, same arguments)
  long long g = (per_rank + bs::kTpThreads - 1) / bs::kTpThreads;
  g = std::min<long long>(g, std::min(d->num_sms, bs::kTpMaxCtas));
  g = std::max<long long>(g, 1);
  cudaGetLastError();
  bs::k_tp_reduce_switch<<<static_cast<int>(g), bs::kTpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      data_mc, static_cast<uint32_t*>(flags), flags_mc, nvec, rank, world, epoch,
      limit_ns ? limit_ns : bs::kWaitLimitNs, d->status);
  return launch_status("k_tp_reduce_switch launch");
}

size_t bs_fp8_workspace_bytes(int M, int N, int K, int fused) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 || N % (fused ? 256 : 128)) return 0;
  DeviceState* d = device_state();
  const int sms = d ? d->num_sms : 148;
  if (M > 128) return prefill_plan(fused != 0, M, N, K, sms).stream_k ? prefill_ws_bytes(sms) : 0;
  const int tiles = fused ? N / 256 : N / 128;
  if (tiles > kMaxDecodeTiles) return 0;
  return decode_ws_bytes(decode_grid(sms, tiles, K / 128), fused ? 2 : 1, ntp_for(M));
}

int bs_fp8_group_quant(const void* x, int ldx, void* A, float* As, int M, int K, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0 || ldx < K || ldx % 8 != 0) return BS_ERR_ARG;
  if (M == 0) return BS_OK;
  if (!x || !A || !As) return BS_ERR_ARG;
  if (!aligned16(x) || !aligned16(A)) return BS_ERR_ALIGN;
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  if (K <= bs::kNormMaxK) {
    // whole rows per CTA, the next row's loads in flight while the current one is quantised
    return launch_row_quant(row_kernel<false, false>(K), d->num_sms, x, ldx, nullptr, K, nullptr, 0.f, A, As, M, K,
                            stream, "k_row_group_quant launch");
  }
  // wider rows: sixteen threads per 128-group, grid-stride over the groups
  const long long groups = static_cast<long long>(M) * (K / 128);
  const int per_block = bs::kQuantThreads / 16;
  long long blocks = (groups + per_block - 1) / per_block;
  const long long cap = static_cast<long long>(d->num_sms) * 16;
  if (blocks > cap) blocks = cap;
  return launch_pdl(bs::k_group_quant, static_cast<int>(blocks), bs::kQuantThreads, 0, static_cast<cudaStream_t>(stream),
                    "k_group_quant launch", static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(A), As,
                    M, K);
}

int bs_fp8_rmsnorm_group_quant(const void* x, int ldx, void* residual, int ldr, const void* weight, float eps,
                               void* A, float* As, int M, int K, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0 || ldx < K || ldx % 8 != 0) return BS_ERR_ARG;
  if (residual && (ldr < K || ldr % 8 != 0)) return BS_ERR_ARG;
  if (!(eps >= 0.f)) return BS_ERR_ARG;
  if (M == 0) return BS_OK;
  if (!x || !weight || !A || !As) return BS_ERR_ARG;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(A) || (residual && !aligned16(residual))) return BS_ERR_ALIGN;
  if (K > bs::kNormMaxK) return BS_ERR_ARG;
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  return launch_row_quant(residual ? row_kernel<true, true>(K) : row_kernel<true, false>(K), d->num_sms, x, ldx,
                          residual, ldr, weight, eps, A, As, M, K, stream, "k_row_group_quant<norm> launch");
}

int bs_fp8_silu_mul(const void* gate_up, int ld_in, void* out, int ld_out, int M, int I, void* stream) {
  if (M < 0 || I <= 0 || I % 8 || ld_in < 2 * I || ld_in % 8 || ld_out < I || ld_out % 8) return BS_ERR_ARG;
  if (M == 0) return BS_OK;
  if (!gate_up || !out) return BS_ERR_ARG;
  if (!aligned16(gate_up) || !aligned16(out)) return BS_ERR_ALIGN;
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  const long long chunks = static_cast<long long>(M) * (I / 8);
  const long long want = (chunks + 255) / 256;
  const int grid = static_cast<int>(want < 4ll * d->num_sms ? want : 4ll * d->num_sms);
  return launch_pdl(bs::k_silu_mul, grid, 256, 0, static_cast<cudaStream_t>(stream), "k_silu_mul launch",
                    static_cast<const __nv_bfloat16*>(gate_up), ld_in, static_cast<__nv_bfloat16*>(out), ld_out, M,
                    I);
}

int bs_fp8_pack_tiles(const void* W, void* tiles, int N, int K, void* stream) {
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return BS_ERR_ARG;
  if (!W || !tiles) return BS_ERR_ARG;
  if (!aligned16(W) || !aligned16(tiles)) return BS_ERR_ALIGN;
  const long long nt = static_cast<long long>(N / 128) * (K / 128);
  if (nt > 0x7fffffffLL) return BS_ERR_ARG;
  cudaGetLastError();
  bs::k_pack_tiles<<<static_cast<int>(nt), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(W), static_cast<uint8_t*>(tiles), N, K);
  return launch_status("k_pack_tiles launch");
}

int bs_fp8_status(int* code, int clear) {
  if (!code) return BS_ERR_ARG;
  if (!device_state()) return BS_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return BS_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bs_status, sizeof(int)) != cudaSuccess) return BS_ERR_CUDA;
  *code = v;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_bs_status, &zero, sizeof(int)) != cudaSuccess) return BS_ERR_CUDA;
  }
  return BS_OK;
}

int bs_fp8_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  DeviceState* d = device_state();
  if (!d) return BS_ERR_CUDA;
  if (limit_ns > 10000000000ull) return BS_ERR_ARG;  // keep the self-test short
  cudaGetLastError();
  k_selftest_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, d->status);
  return launch_status("k_selftest_wait launch");
}

int bs_fp8_launch_plan(int M, int N, int K, int fused, int* plan, int n) {
  if (!plan || n < BS_PLAN_FIELDS) return BS_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 || N % (fused ? 256 : 128)) return BS_ERR_ARG;
  for (int i = 0; i < n; ++i) plan[i] = 0;
  DeviceState* d = device_state();
  const int sms = d ? d->num_sms : 148;
  const int KB = K / 128;
  if (M <= 128) {
    const int ntp = ntp_for(M);
    const int tiles = fused ? N / 256 : N / 128;
    int split = 0;
    const int grid = decode_grid(sms, tiles, KB, &split);
    int cfg[5];
    if (!(fused ? decode_cfg_values<true>(ntp, cfg) : decode_cfg_values<false>(ntp, cfg))) return BS_ERR_ARG;
    plan[BS_PLAN_KIND] = 1;
    plan[BS_PLAN_TILE_ROWS] = 128;  // weight rows (swap-AB: the weights are the MMA's M side)
    plan[BS_PLAN_TILE_COLS] = ntp;  // tokens, padded to a multiple of 16
    plan[BS_PLAN_STAGES] = cfg[0];
    plan[BS_PLAN_THREADS] = cfg[1];
    plan[BS_PLAN_GRID] = grid;
    plan[BS_PLAN_CLUSTER] = 1;
    plan[BS_PLAN_TMEM_COLS] = cfg[2];
    plan[BS_PLAN_SPLIT] = split;
    plan[BS_PLAN_WARPGROUPS] = cfg[3];
    plan[BS_PLAN_SMEM] = cfg[4];
    return BS_OK;
  }
  const PrefillPlan pl = prefill_plan(fused != 0, M, N, K, sms);
  const int tiles = pl.num_m * pl.num_n;
  plan[BS_PLAN_KIND] = 2;
  plan[BS_PLAN_SPLIT] = pl.stream_k ? -1 : 0;  // stream-K needs the workspace bs_fp8_workspace_bytes reports
  plan[BS_PLAN_TILE_ROWS] = pl.rows;
  plan[BS_PLAN_TILE_COLS] = 256;
  if (pl.pair) {
    plan[BS_PLAN_STAGES] = fused ? bs::PrefillCfg<true, true>::kStages : bs::PrefillCfg<false, true>::kStages;
    plan[BS_PLAN_SMEM] = fused ? bs::PrefillCfg<true, true>::kSmemBytes : bs::PrefillCfg<false, true>::kSmemBytes;
    const int pairs = (sms / 2 < tiles) ? sms / 2 : tiles;
    plan[BS_PLAN_GRID] = 2 * pairs;
    plan[BS_PLAN_CLUSTER] = 2;
  } else {
    plan[BS_PLAN_STAGES] = fused ? bs::PrefillCfg<true, false>::kStages : bs::PrefillCfg<false, false>::kStages;
    plan[BS_PLAN_SMEM] = fused ? bs::PrefillCfg<true, false>::kSmemBytes : bs::PrefillCfg<false, false>::kSmemBytes;
    plan[BS_PLAN_GRID] = tiles < sms ? tiles : sms;
    plan[BS_PLAN_CLUSTER] = 1;
  }
  plan[BS_PLAN_THREADS] = bs::PrefillCfg<false, false>::kThreads;
  plan[BS_PLAN_GROUP_M] = pl.group_m;
  plan[BS_PLAN_TMEM_COLS] = bs::PrefillCfg<false, false>::kTmemCols;
  plan[BS_PLAN_WARPGROUPS] = 2;
  plan[BS_PLAN_TILES] = tiles;
  return BS_OK;
}

int bs_fp8_num_sms(void) {
  DeviceState* d = device_state();
  return d ? d->num_sms : 0;
}

const char* bs_fp8_error_string(int code) {
  switch (code) {
    case BS_OK: return "ok";
    case BS_ERR_ARG: return "argument outside the contract (shape, stride or dtype)";
    case BS_ERR_ALIGN: return "pointer or row stride not 16-byte aligned";
    case BS_ERR_WORKSPACE: return "workspace missing or too small";
    case BS_ERR_TMAP: return "TMA descriptor could not be created";
    case BS_ERR_CUDA: return "CUDA runtime call failed";
    case BS_ERR_BUILD: return "kernel register count does not match its setmaxnreg split; refusing to launch";
    case BS_ERR_SCRATCH: return "shape needs more split-K scratch than bs_fp8_gemm_noalloc's fixed 4 MiB array";
    case BS_ERR_TIMEOUT_FULL: return "device: bounded wait for a TMA stage ran out";
    case BS_ERR_TIMEOUT_EMPTY: return "device: bounded wait for a free stage ran out";
    case BS_ERR_TIMEOUT_PFULL: return "device: bounded wait for an MMA partial ran out";
    case BS_ERR_TIMEOUT_PEMPTY: return "device: bounded wait for a TMEM buffer ran out";
    case BS_ERR_TIMEOUT_DRAIN: return "device: teardown drain ran out";
    case BS_ERR_TIMEOUT_SELFTEST: return "device: self-test wait ran out (expected)";
    default: return "unknown status code";
  }
}

int bs_fp8_abi_version(void) { return 1; }

const char* bs_fp8_last_cuda_error(void) { return g_last_cuda_error; }

#ifdef BS_TRACE
// Profiling builds only (-DBS_TRACE): copies and clears the stage counters of the current device.
int bs_fp8_trace_read(unsigned long long* out, int n) {
  if (!out || n <= 0 || n > 64) return BS_ERR_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return BS_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, bs::g_bs_trace, sizeof(unsigned long long) * n) != cudaSuccess) return BS_ERR_CUDA;
  unsigned long long zero[64] = {0};
  if (cudaMemcpyToSymbol(bs::g_bs_trace, zero, sizeof(zero)) != cudaSuccess) return BS_ERR_CUDA;
  return BS_OK;
}
#endif

}  // extern "C"
