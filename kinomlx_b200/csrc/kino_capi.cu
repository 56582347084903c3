// Host side of libkino_b200.so: argument checks, TMA descriptor encoding and launches for the
// extern "C" entry points declared in include/kino.h. One translation unit holds every kernel so
// the device error word is a single symbol without relocatable device code.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "../../include/kino.h"
#include "kino_attention.cuh"
#include "kino_common.cuh"
#include "kino_gemm.cuh"
#include "kino_conv3d.cuh"
#include "kino_ops.cuh"
#include "kino_peer.cuh"
#include "kino_sol.cuh"
#include "kino_na.cuh"
#include "kino_diffusion.cuh"
#include "kino_vae.cuh"
#include "kino_quant.cuh"
#include "kino_f32.cuh"

// Scratch of kino_group_norm_noalloc: a fixed device array that every GPU loading this library
// holds until the process exits. Host code only sees a stand-in symbol for it, so its device
// address is looked up once per device (cudaGetSymbolAddress, with that device current) and
// passed to the kernels like any workspace pointer.
static __device__ __align__(256) unsigned char g_group_norm_scratch[KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local char g_err[512] = {0};

kino_status fail(kino_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

thread_local cudaError_t t_launch_error = cudaSuccess;

kino_status check_launch(const char* what) {
  cudaError_t e = t_launch_error;
  t_launch_error = cudaSuccess;
  const cudaError_t last = cudaGetLastError();
  if (e == cudaSuccess) e = last;
  if (e != cudaSuccess) return fail(KINO_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return KINO_OK;
}

// Programmatic dependent launch (the kernel's prologue may overlap the previous kernel's tail;
// every kernel waits with griddepcontrol.wait before touching global memory) unless
// KINO_PDL=0 in the environment.
bool pdl_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("KINO_PDL");
    enabled = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return enabled == 1;
}

// Launch with the PDL attribute (and a cluster of `cluster_x` CTAs when > 1); a failure is
// reported by the next check_launch().
template <typename... KArgs, typename... Args>
void launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess && t_launch_error == cudaSuccess) t_launch_error = e;
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                Args&&... args) {
  launch_ex(kernel, grid, block, smem, stream, 1, std::forward<Args>(args)...);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- driver entry point for TMA
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 tensor map, dims innermost first, strides in elements for dims 1.., box sizes.
kino_status make_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_elems, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(KINO_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base)) return fail(KINO_EINVAL, "TMA base address not 16-byte aligned");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    s[i] = strides_elems[i] * 2;
    if (s[i] % 16 != 0) return fail(KINO_EINVAL, "TMA stride %llu bytes not a multiple of 16",
                                    static_cast<unsigned long long>(s[i]));
  }
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s,
                        b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KINO_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KINO_OK;
}

int device_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Opt a kernel into its dynamic shared memory once per device.
template <typename K>
kino_status ensure_smem(K kernel, int bytes, int slot) {
  static bool done[32][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[slot][dev]) return KINO_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(KINO_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[slot][dev] = true;
  return KINO_OK;
}

template <int BN, int STAGES>
kino_status launch_gemm(const void* x, const void* w, void* out, const kino::GemmShape& s0,
                        int64_t ldx, int64_t bsx, int64_t ldw, const kino::GemmEpi& e,
                        cudaStream_t stream, int slot, const void* w_lead, int64_t ldw_lead) {
  using L = kino::GemmSmem<BN, STAGES>;
  CUtensorMap ma, mb, mbl;
  const uint64_t da[3] = {static_cast<uint64_t>(s0.k), static_cast<uint64_t>(s0.m),
                          static_cast<uint64_t>(s0.batch)};
  const uint64_t sa[2] = {static_cast<uint64_t>(ldx),
                          static_cast<uint64_t>(s0.batch > 1 ? bsx : ldx * s0.m)};
  const uint32_t ba[3] = {64, 128, 1};
  kino_status st = make_map(&ma, x, 3, da, sa, ba);
  if (st != KINO_OK) return st;
  const uint64_t db[2] = {static_cast<uint64_t>(s0.k), static_cast<uint64_t>(s0.n)};
  const uint64_t sb[1] = {static_cast<uint64_t>(ldw)};
  const uint32_t bb[2] = {64, static_cast<uint32_t>(BN)};
  st = make_map(&mb, w, 2, db, sb, bb);
  if (st != KINO_OK) return st;
  mbl = mb;
  if (w_lead != nullptr) {
    const uint64_t sbl[1] = {static_cast<uint64_t>(ldw_lead)};
    st = make_map(&mbl, w_lead, 2, db, sbl, bb);
    if (st != KINO_OK) return st;
  }
  kino::GemmShape s = s0;
  s.tiles_m = (s.m + kino::GEMM_BM - 1) / kino::GEMM_BM;
  s.tiles_n = (s.n + BN - 1) / BN;
  s.num_tiles = s.tiles_m * s.tiles_n * s.batch;
  s.kblocks = (s.k + kino::GEMM_BK - 1) / kino::GEMM_BK;
  auto kernel = kino::gemm_bf16_tc_kernel<BN, STAGES>;
  st = ensure_smem(kernel, L::TOTAL, slot);
  if (st != KINO_OK) return st;
  const int grid = s.num_tiles < device_sms() ? s.num_tiles : device_sms();
  launch_pdl(kernel, dim3(grid), dim3(kino::GEMM_THREADS), L::TOTAL, stream,
      ma, mb, mbl, reinterpret_cast<__nv_bfloat16*>(out), s, e);
  return check_launch("kino_linear");
}

// Split-K workspace of the single-SM conv: tile counters first (one int per tile and lane
// quarter), then the fp32 partial sums.
#ifndef KINO_CONV_SPLIT_K
#define KINO_CONV_SPLIT_K 1
#endif
constexpr int64_t KINO_CONV_SPLIT_COUNTERS_BYTES = 16384;
constexpr int64_t KINO_CONV_SPLIT_WORKSPACE_BYTES = KINO_CONV_SPLIT_COUNTERS_BYTES + (48ll << 20);

template <int BN, int STAGES, int MT>
kino_status launch_conv(const kino_conv3d_args* a, const kino::ConvShape& s0, cudaStream_t stream,
                        int slot) {
  using L = kino::ConvSmem<BN, STAGES, MT>;
  CUtensorMap mx, mw;
  const uint64_t dx[4] = {static_cast<uint64_t>(s0.Cin), static_cast<uint64_t>(s0.W),
                          static_cast<uint64_t>(s0.H), static_cast<uint64_t>(s0.F)};
  const uint64_t sx[3] = {static_cast<uint64_t>(s0.Cin), static_cast<uint64_t>(s0.W) * s0.Cin,
                          static_cast<uint64_t>(s0.H) * s0.W * s0.Cin};
  const uint32_t bx[4] = {64, static_cast<uint32_t>(s0.tw), static_cast<uint32_t>(s0.th), 1};
  kino_status st = make_map(&mx, a->x, 4, dx, sx, bx);
  if (st != KINO_OK) return st;
  const uint64_t k = 27ull * s0.Cin;
  const uint64_t dw[2] = {k, static_cast<uint64_t>(s0.N)};
  const uint64_t sw[1] = {k};
  const uint32_t bw[2] = {64, static_cast<uint32_t>(BN)};
  st = make_map(&mw, a->weight, 2, dw, sw, bw);
  if (st != KINO_OK) return st;
  kino::ConvShape s = s0;
  s.tiles_m = (s.boxes + MT - 1) / MT;
  s.tiles_n = (s.N + BN - 1) / BN;
  s.splits = 1;
  s.kper = s.kblocks;
  kino::ConvEpi e;
  e.split_count = nullptr;
  e.split_partial = nullptr;
  // Split-K when the output tiles fill less than half of the SMs and the caller gave a
  // workspace: at least 32 K blocks per split (below that the partial sums' round trip costs
  // more than the idle SMs), at most 8 splits, partials within the workspace.
  const int64_t tiles = static_cast<int64_t>(s.tiles_m) * s.tiles_n;
  if (KINO_CONV_SPLIT_K && MT == 1 && a->workspace != nullptr && 2 * tiles <= device_sms() &&
      4 * tiles * 4 <= KINO_CONV_SPLIT_COUNTERS_BYTES) {
    int splits = static_cast<int>(device_sms() / tiles);
    if (splits > 8) splits = 8;
    if (splits > s.kblocks / 32) splits = s.kblocks / 32;
    while (splits > 1 && KINO_CONV_SPLIT_COUNTERS_BYTES + tiles * splits * 128 * BN * 4 >
                              a->workspace_bytes)
      --splits;
    if (splits > 1) {
      s.kper = (s.kblocks + splits - 1) / splits;
      s.splits = (s.kblocks + s.kper - 1) / s.kper;
      e.split_count = static_cast<int*>(a->workspace);
      e.split_partial = reinterpret_cast<float*>(static_cast<char*>(a->workspace) +
                                                 KINO_CONV_SPLIT_COUNTERS_BYTES);
    }
  }
  s.num_tiles = s.tiles_m * s.tiles_n * s.splits;
  auto kernel = kino::conv3d_tc_kernel<BN, STAGES, MT>;
  st = ensure_smem(kernel, L::TOTAL, slot);
  if (st != KINO_OK) return st;
  const int grid = s.num_tiles < device_sms() ? s.num_tiles : device_sms();
  e.bias = static_cast<const __nv_bfloat16*>(a->bias);
  e.residual = static_cast<const __nv_bfloat16*>(a->residual);
  e.stats = static_cast<float*>(a->stats);
  e.group_size = s.Co / kino::GN_GROUPS;
  if (e.stats != nullptr && grid * 4 > a->stats_records)
    return fail(KINO_EINVAL, "kino_conv3d: statistics buffer holds %lld records, %d needed",
                (long long)a->stats_records, grid * 4);
  launch_pdl(kernel, dim3(grid), dim3(kino::CONV_THREADS), L::TOTAL, stream,
      mx, mw, static_cast<__nv_bfloat16*>(a->out), s, e);
  return check_launch("kino_conv3d");
}

template <int BN, int STAGES, int KSUB, int HALO = 0>
kino_status launch_conv_2sm(const kino_conv3d_args* a, const kino::ConvShape& s0,
                            cudaStream_t stream, int slot) {
  using L = kino::ConvPairSmem<BN, STAGES, KSUB, HALO>;
  CUtensorMap mx, mw;
  const uint64_t dx[4] = {static_cast<uint64_t>(s0.Cin), static_cast<uint64_t>(s0.W),
                          static_cast<uint64_t>(s0.H), static_cast<uint64_t>(s0.F)};
  const uint64_t sx[3] = {static_cast<uint64_t>(s0.Cin), static_cast<uint64_t>(s0.W) * s0.Cin,
                          static_cast<uint64_t>(s0.H) * s0.W * s0.Cin};
  // HALO 1: one 128-voxel row plus a voxel on each side per load; 2: th + 2 rows of tw
  const uint32_t bx[4] = {64, static_cast<uint32_t>(HALO == 1 ? kino::CONV_HALO_ROWS : s0.tw),
                          static_cast<uint32_t>(HALO == 2 ? s0.th + 2 : s0.th), 1};
  kino_status st = make_map(&mx, a->x, 4, dx, sx, bx);
  if (st != KINO_OK) return st;
  const uint64_t k = 27ull * s0.Cin;
  const uint64_t dw[2] = {k, static_cast<uint64_t>(s0.N)};
  const uint64_t sw[1] = {k};
  const uint32_t bw[2] = {64, static_cast<uint32_t>(BN / 2)};
  st = make_map(&mw, a->weight, 2, dw, sw, bw);
  if (st != KINO_OK) return st;
  kino::ConvShape s = s0;
  s.tiles_m = (s.boxes + 1) / 2;
  s.tiles_n = (s.N + BN - 1) / BN;
  s.num_tiles = s.tiles_m * s.tiles_n;
  s.splits = 1;
  s.kper = s.kblocks;
  auto kernel = kino::conv3d_2sm_kernel<BN, STAGES, KSUB, HALO>;
  st = ensure_smem(kernel, L::TOTAL, slot);
  if (st != KINO_OK) return st;
  const int max_pairs = device_sms() / 2;
  const int pairs = s.num_tiles < max_pairs ? s.num_tiles : max_pairs;
  kino::ConvEpi e;
  e.bias = static_cast<const __nv_bfloat16*>(a->bias);
  e.residual = static_cast<const __nv_bfloat16*>(a->residual);
  e.stats = static_cast<float*>(a->stats);
  e.group_size = s.Co / kino::GN_GROUPS;
  e.split_count = nullptr;
  e.split_partial = nullptr;
  if (e.stats != nullptr && 2 * pairs * 4 > a->stats_records)
    return fail(KINO_EINVAL, "kino_conv3d: statistics buffer holds %lld records, %d needed",
                (long long)a->stats_records, 2 * pairs * 4);
  launch_ex(kernel, dim3(2 * pairs), dim3(kino::CONV_PAIR_THREADS), L::TOTAL, stream, 2, mx, mw,
            static_cast<__nv_bfloat16*>(a->out), s, e);
  return check_launch("kino_conv3d (2-SM)");
}

template <int STAGES>
kino_status launch_gemm_2sm(const void* x, const void* w, void* out, const kino::GemmShape& s0,
                            int64_t ldx, int64_t bsx, int64_t ldw, const kino::GemmEpi& e,
                            cudaStream_t stream, int slot, const void* w_lead, int64_t ldw_lead) {
  using L = kino::Gemm2SmSmem<STAGES>;
  CUtensorMap ma, mb, mbl;
  const uint64_t da[3] = {static_cast<uint64_t>(s0.k), static_cast<uint64_t>(s0.m),
                          static_cast<uint64_t>(s0.batch)};
  const uint64_t sa[2] = {static_cast<uint64_t>(ldx),
                          static_cast<uint64_t>(s0.batch > 1 ? bsx : ldx * s0.m)};
  const uint32_t ba[3] = {64, 128, 1};
  kino_status st = make_map(&ma, x, 3, da, sa, ba);
  if (st != KINO_OK) return st;
  const uint64_t db[2] = {static_cast<uint64_t>(s0.k), static_cast<uint64_t>(s0.n)};
  const uint64_t sb[1] = {static_cast<uint64_t>(ldw)};
  const uint32_t bb[2] = {64, 128};
  st = make_map(&mb, w, 2, db, sb, bb);
  if (st != KINO_OK) return st;
  mbl = mb;
  if (w_lead != nullptr) {
    const uint64_t sbl[1] = {static_cast<uint64_t>(ldw_lead)};
    st = make_map(&mbl, w_lead, 2, db, sbl, bb);
    if (st != KINO_OK) return st;
  }
  kino::GemmShape s = s0;
  s.tiles_m = (s.m + 255) / 256;
  s.tiles_n = (s.n + 255) / 256;
  s.num_tiles = s.tiles_m * s.tiles_n * s.batch;
  s.kblocks = (s.k + kino::GEMM_BK - 1) / kino::GEMM_BK;
  auto kernel = kino::gemm_bf16_2sm_kernel<STAGES>;
  st = ensure_smem(kernel, L::TOTAL, slot);
  if (st != KINO_OK) return st;
  const int max_pairs = device_sms() / 2;
  const int pairs = s.num_tiles < max_pairs ? s.num_tiles : max_pairs;
  launch_ex(kernel, dim3(2 * pairs, 1, 1), dim3(kino::GEMM_THREADS, 1, 1), L::TOTAL, stream, 2, ma,
            mb, mbl, reinterpret_cast<__nv_bfloat16*>(out), s, e);
  return check_launch("kino_linear (2-SM)");
}

// Pipeline depth of the CTA-pair GEMM (32 KiB per stage per CTA; 7 is the most that fits).
#ifndef KINO_GEMM_PAIR_STAGES
#define KINO_GEMM_PAIR_STAGES 7
#endif

// CTA-pair GEMM tiles unless KINO_GEMM_PAIRS=0 in the environment (kept for A/B measurements).
bool gemm_pairs_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("KINO_GEMM_PAIRS");
    enabled = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return enabled == 1;
}

// Tile shape of a product: 1 = CTA pairs with 256 x 256 tiles, 2 = one SM with 128 x 256 tiles,
// 3 = one SM with 128 x 128 tiles. The persistent kernels run ceil(tiles / slots) waves of
// equal-length tiles, so the estimate is waves x tile time, the tile time relative to the
// CTA-pair kernel's per-SM share (128 x 256) with the single-SM kernels' measured throughput
// ratios (per mille). The 128 x 128 ratio comes from the small-row products of the
// sequence-parallel ranks (576 and 1152 rows, K = 3072 to 15360, each tiling timed): at 770 the
// estimate picks the fastest tiling for all twelve shapes timed (at 860 it gave 1152 x 9216 to
// the 128 x 128 tiles, 60.7 us, against the pairs' 56.0).
#ifndef KINO_GEMM_E1
#define KINO_GEMM_E1 930
#endif
#ifndef KINO_GEMM_E1B
#define KINO_GEMM_E1B 770
#endif
#ifndef KINO_GEMM_FORCE
#define KINO_GEMM_FORCE 0
#endif
int gemm_tiling(int64_t batch, int64_t m, int64_t n) {
  if (KINO_GEMM_FORCE != 0) return KINO_GEMM_FORCE;
  if (n <= 128) return 3;
  const int64_t sms = device_sms();
  auto waves = [&](int64_t tiles, int64_t slots) { return (tiles + slots - 1) / slots; };
  const int64_t t2 = batch * ((m + 255) / 256) * ((n + 255) / 256);
  const int64_t t1 = batch * ((m + 127) / 128) * ((n + 255) / 256);
  const int64_t t3 = batch * ((m + 127) / 128) * ((n + 127) / 128);
  const double e2 = gemm_pairs_enabled() ? waves(t2, sms / 2) * 1000.0 : 1e30;
  const double e1 = waves(t1, sms) * 1000.0 * 1000.0 / KINO_GEMM_E1;
  const double e3 = waves(t3, sms) * 500.0 * 1000.0 / KINO_GEMM_E1B;
  if (e2 <= e1 && e2 <= e3) return 1;
  return e1 <= e3 ? 2 : 3;
}

// Grid of the GroupNorm apply pass: one resident wave at most, so that the grid-stride loop
// gives every CTA the same share.
int64_t gn_apply_blocks(int64_t voxels, int64_t channels) {
  static int resident = 0;
  if (resident == 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kino::group_norm_apply_kernel, 256,
                                                      0) != cudaSuccess || per_sm < 1)
      per_sm = 2;
    resident = per_sm;
  }
  const int64_t rows_per_cta = 256 / (channels / 8);
  const int64_t blocks = (voxels + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = static_cast<int64_t>(device_sms()) * resident;
  return blocks < cap ? blocks : cap;
}

int gn_parts(int64_t voxels) {
  int64_t p = (voxels + 31) / 32;
  return static_cast<int>(p < 592 ? (p < 1 ? 1 : p) : 592);
}

// The id of the calling thread's current context (cuCtxGetId through the runtime's driver entry
// point), or 0 when there is none or the driver lacks the call. A device reset destroys the
// primary context and the module with it, so a cached symbol address is only valid for the
// context it was looked up in.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  void* ctx = nullptr;
  if (get_current(&ctx) != 0 || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == 0 ? id : 0;
}

// Device address of g_group_norm_scratch for the current device, looked up with that device
// current the first time a context uses it and cached per device with the context's id; a new
// context on the device (after cudaDeviceReset) looks it up again.
void* group_norm_scratch_address(kino_status* status) {
  static std::mutex lock;
  static void* addresses[64] = {nullptr};
  static unsigned long long contexts[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *status = fail(KINO_ECUDA, "kino_group_norm_noalloc: no current device (%s)",
                   cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> guard(lock);
  const unsigned long long ctx = current_context_id();
  if (addresses[dev] == nullptr || ctx == 0 || ctx != contexts[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_group_norm_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = fail(KINO_ECUDA, "kino_group_norm_noalloc: cudaGetSymbolAddress failed (%s)",
                     cudaGetErrorString(e));
      return nullptr;
    }
    addresses[dev] = p;
    contexts[dev] = current_context_id();  // the lookup made the primary context current
  }
  *status = KINO_OK;
  return addresses[dev];
}

}  // namespace

// Sol-Attn workspace sections (all 256-byte aligned), in order.
namespace {

struct SolLayout {
  int64_t nb, words, ncta, width;
  int64_t q16, k16, v16, qmean, kmean, vmean, bits, lists, counts, total;
};

SolLayout sol_layout(int64_t tokens, int64_t heads) {
  SolLayout l;
  l.nb = (tokens + kino::SOL_BLOCK - 1) / kino::SOL_BLOCK;
  l.words = (l.nb + 31) / 32;
  l.ncta = (l.nb + kino::SOL_QBLOCKS - 1) / kino::SOL_QBLOCKS;
  l.width = heads * 128;
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  int64_t at = 0;
  auto take = [&](int64_t bytes) {
    const int64_t here = at;
    at += up(bytes);
    return here;
  };
  l.q16 = take(tokens * l.width * 2);
  l.k16 = take(tokens * l.width * 2);
  l.v16 = take(tokens * l.width * 2);
  l.qmean = take(heads * l.nb * 128 * 4);
  l.kmean = take(heads * l.nb * 128 * 2);
  l.vmean = take(heads * l.nb * 128 * 2);
  l.bits = take(heads * l.nb * l.words * 4);
  l.lists = take(heads * l.ncta * l.nb * 4);
  l.counts = take(heads * l.ncta * 4);
  l.total = at;
  return l;
}

}  // namespace

extern "C" {

int kino_abi_version(void) { return 15; }

const char* kino_last_error(void) { return g_err; }

int kino_num_sms(void) { return device_sms(); }

kino_status kino_device_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(KINO_ECUDA, "stream sync: %s", cudaGetErrorString(e));
  int flag = 0;
  e = cudaMemcpyFromSymbol(&flag, kino::g_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(KINO_ECUDA, "device status: %s", cudaGetErrorString(e));
  if (flag != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(kino::g_device_error, &zero, sizeof(int));
    if (flag == KINO_ETIMEOUT) return fail(flag, "a kernel wait timed out (device status %d)", flag);
    return fail(flag, "a kernel skipped an out-of-range index (device status %d)", flag);
  }
  return KINO_OK;
}

kino_status kino_linear(const void* x, const void* w, void* out, int64_t batch, int64_t m,
                        int64_t n, int64_t k, int64_t ldx, int64_t bsx, int64_t ldw, int64_t ldo,
                        int64_t bso, const kino_epilogue* epi, void* stream) {
  if (x == nullptr || w == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_linear: null operand");
  if (batch < 1 || m < 1 || n < 1 || k < 1) return fail(KINO_EINVAL, "kino_linear: empty shape");
  if (k % 8 || n % 8 || ldx % 8 || ldw % 8 || ldo % 8 || (batch > 1 && (bsx % 8 || bso % 8)))
    return fail(KINO_ENOTSUPPORTED,
                "kino_linear: k, n and strides must be multiples of 8 (k=%lld n=%lld)",
                (long long)k, (long long)n);
  const bool swiglu = epi != nullptr && epi->kind == kino::EPI_SWIGLU;
  const int64_t n_out = swiglu ? epi->act_col_begin + (n - epi->act_col_begin) / 2 : n;
  if (ldx < k || ldw < k || ldo < n_out)
    return fail(KINO_EINVAL, "kino_linear: stride below width");
  if (swiglu && (epi->act_col_begin % 32 || (n - epi->act_col_begin) % 32 || epi->act_col_begin < 0))
    return fail(KINO_ENOTSUPPORTED, "kino_linear: SwiGLU columns must come in blocks of 32");
  if (m > (1 << 30) || n > (1 << 30) || k > (1 << 30) || batch > 65535)
    return fail(KINO_ENOTSUPPORTED, "kino_linear: shape too large");
  if (!aligned16(out)) return fail(KINO_EINVAL, "kino_linear: out not 16-byte aligned");
  kino::GemmEpi e;
  std::memset(&e, 0, sizeof(e));
  e.kind = kino::EPI_NONE;
  e.act_col_begin = 0;
  if (epi != nullptr) {
    e.kind = epi->kind;
    e.bias = static_cast<const __nv_bfloat16*>(epi->bias);
    e.residual = static_cast<const __nv_bfloat16*>(epi->residual);
    e.ld_res = epi->ld_residual;
    e.bs_res = epi->bs_residual;
    e.gate = static_cast<const __nv_bfloat16*>(epi->gate);
    e.bs_gate = epi->bs_gate;
    e.act_col_begin = epi->act_col_begin;
    e.scalar = epi->scalar;
    e.aux = static_cast<const __nv_bfloat16*>(epi->aux);
    e.ld_aux = epi->ld_aux;
    e.bs_aux = epi->bs_aux;
    e.scalar2 = epi->scalar2;
    if (e.kind < 0 || e.kind > 6) return fail(KINO_EINVAL, "kino_linear: unknown epilogue");
    if (e.bias != nullptr && !aligned16(e.bias))
      return fail(KINO_EINVAL, "kino_linear: bias not 16-byte aligned");
    if (e.kind == kino::EPI_GATED_RESIDUAL &&
        (e.residual == nullptr || e.gate == nullptr || !aligned16(e.residual) ||
         !aligned16(e.gate) || e.ld_res % 8 || e.bs_res % 8 || e.bs_gate % 8))
      return fail(KINO_EINVAL, "kino_linear: gated residual needs aligned residual and gate");
    if ((e.kind == kino::EPI_EULER || e.kind == kino::EPI_EULER_X0) &&
        (e.aux == nullptr || !aligned16(e.aux) || e.ld_aux % 8 || e.bs_aux % 8))
      return fail(KINO_EINVAL, "kino_linear: Euler epilogue needs an aligned sample");
    for (int r = 0; r < 2; ++r) {
      e.norm_w[r] = static_cast<const __nv_bfloat16*>(epi->norm_weight[r]);
      e.norm_col[r] = epi->norm_col[r];
    }
    e.norm_width = epi->norm_width;
    e.rope_cos = epi->rope_cos;
    e.rope_sin = epi->rope_sin;
    e.rope_rows = epi->rope_rows;
    e.rope_offset = epi->rope_offset;
    e.rope_batched = epi->rope_batched;
    e.norm_eps = epi->norm_eps;
    if (e.norm_w[0] != nullptr || e.norm_w[1] != nullptr) {
      if (e.rope_cos == nullptr || e.rope_sin == nullptr || !aligned16(e.rope_cos) ||
          !aligned16(e.rope_sin) || e.norm_width <= 0 || e.norm_width % 128)
        return fail(KINO_EINVAL, "kino_linear: QK norm needs 128-wide heads and aligned tables");
      for (int r = 0; r < 2; ++r)
        if (e.norm_w[r] != nullptr &&
            (!aligned16(e.norm_w[r]) || e.norm_col[r] % 128 || e.norm_col[r] < 0 ||
             e.norm_col[r] + e.norm_width > n))
          return fail(KINO_EINVAL, "kino_linear: QK norm range outside the product");
      if (e.rope_offset < 0 || e.rope_offset + m > e.rope_rows)
        return fail(KINO_EINVAL, "kino_linear: RoPE table shorter than the rows");
      if (e.kind == kino::EPI_SWIGLU &&
          ((e.norm_w[0] && e.norm_col[0] + e.norm_width > e.act_col_begin) ||
           (e.norm_w[1] && e.norm_col[1] + e.norm_width > e.act_col_begin)))
        return fail(KINO_EINVAL, "kino_linear: QK norm ranges must precede the SwiGLU columns");
    }
  }
  if (epi != nullptr && epi->scatter_ptrs != nullptr) {
    const int64_t pw = epi->part_width, sw = epi->seg_width, sc = epi->scatter_cols;
    if (batch != 1) return fail(KINO_EINVAL, "kino_linear: scatter needs batch 1");
    if (epi->world < 1 || epi->world > kino::PEER_MAX_WORLD)
      return fail(KINO_EINVAL, "kino_linear: scatter world 1..%d", kino::PEER_MAX_WORLD);
    if (pw <= 0 || pw % 128 || sw <= 0 || sw % pw || sw / pw != epi->world || sc <= 0 ||
        sc % sw || sc / sw > 4 || sc > n || (swiglu && sc > epi->act_col_begin))
      return fail(KINO_EINVAL, "kino_linear: scatter segments must split into world parts of "
                               "128-column heads and precede the other columns");
    if (epi->scatter_ld % 8 || epi->scatter_row0 < 0 || epi->scatter_row0 + m > epi->scatter_rows)
      return fail(KINO_EINVAL, "kino_linear: scatter rows outside the receive buffers");
    for (int64_t g = 0; g < sc / sw; ++g)
      if (epi->seg_slot[g] < 0 || (epi->seg_slot[g] + 1) * pw > epi->scatter_ld)
        return fail(KINO_EINVAL, "kino_linear: scatter slot outside the receive row");
    e.scatter_ptrs = reinterpret_cast<__nv_bfloat16* const*>(epi->scatter_ptrs);
    e.scatter_cols = static_cast<int>(sc);
    e.seg_width = static_cast<int>(sw);
    e.part_width = static_cast<int>(pw);
    e.scatter_ld = epi->scatter_ld;
    e.scatter_row0 = epi->scatter_row0;
    for (int g = 0; g < 4; ++g) e.seg_slot[g] = epi->seg_slot[g];
  }
  if (epi != nullptr && epi->bias_after_round) {
    if (e.norm_w[0] != nullptr || e.norm_w[1] != nullptr)
      return fail(KINO_ENOTSUPPORTED, "kino_linear: bias after rounding is not combined with the "
                                      "fused QK norm");
    e.bias_after_round = 1;
  }
  const void* w_lead = nullptr;
  int64_t ldw_lead = 0;
  e.lead_rows = 0;
  if (epi != nullptr && epi->lead_rows > 0) {
    if (epi->lead_rows % 256 || epi->lead_rows >= m || epi->w_lead == nullptr ||
        !aligned16(epi->w_lead) || epi->ldw_lead % 8 || epi->ldw_lead < k)
      return fail(KINO_EINVAL, "kino_linear: lead rows need a multiple of 256 below m and an "
                               "aligned lead weight");
    for (int r = 0; r < 2; ++r)
      if ((e.norm_w[r] != nullptr) != (epi->norm_weight_lead[r] != nullptr) ||
          (epi->norm_weight_lead[r] != nullptr && !aligned16(epi->norm_weight_lead[r])))
        return fail(KINO_EINVAL, "kino_linear: lead rows need QK norm weights like the others");
    if (e.kind == kino::EPI_GATED_RESIDUAL &&
        (epi->gate_lead == nullptr || !aligned16(epi->gate_lead)))
      return fail(KINO_EINVAL, "kino_linear: lead rows need their own aligned gate");
    w_lead = epi->w_lead;
    ldw_lead = epi->ldw_lead;
    e.lead_rows = static_cast<int>(epi->lead_rows);
    for (int r = 0; r < 2; ++r)
      e.norm_w_lead[r] = static_cast<const __nv_bfloat16*>(epi->norm_weight_lead[r]);
    e.gate_lead = static_cast<const __nv_bfloat16*>(epi->gate_lead);
  }
  kino::GemmShape s;
  std::memset(&s, 0, sizeof(s));
  s.batch = static_cast<int>(batch);
  s.m = static_cast<int>(m);
  s.n = static_cast<int>(n);
  s.k = static_cast<int>(k);
  s.ldo = ldo;
  s.bs_out = batch > 1 ? bso : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (gemm_tiling(batch, m, n)) {
    case 1:
      return launch_gemm_2sm<KINO_GEMM_PAIR_STAGES>(x, w, out, s, ldx, bsx, ldw, e, st, 6, w_lead,
                                                    ldw_lead);
    case 2:
      return launch_gemm<256, 4>(x, w, out, s, ldx, bsx, ldw, e, st, 1, w_lead, ldw_lead);
    default:
      return launch_gemm<128, 6>(x, w, out, s, ldx, bsx, ldw, e, st, 0, w_lead, ldw_lead);
  }
}

kino_status kino_gemv(const void* x, int64_t ldx, const void* w, const void* bias, void* y,
                      int64_t ldy, int64_t batch, int64_t n, int64_t k, int act, void* stream) {
  if (x == nullptr || w == nullptr || y == nullptr) return fail(KINO_EINVAL, "kino_gemv: null");
  if (batch < 1 || batch > kino::GEMV_MAXB)
    return fail(KINO_ENOTSUPPORTED, "kino_gemv: batch must be 1..%d", kino::GEMV_MAXB);
  if (k % 8 || !aligned16(w) || n < 1 || k < 8)
    return fail(KINO_ENOTSUPPORTED, "kino_gemv: k %% 8 and aligned weight required");
  const int smem = static_cast<int>(batch * k * sizeof(float));
  if (smem > 200 * 1024) return fail(KINO_ENOTSUPPORTED, "kino_gemv: k too large");
  kino_status s = ensure_smem(kino::gemv_kernel, 200 * 1024, 2);
  if (s != KINO_OK) return s;
  const int per = kino::GEMV_THREADS / 32;
  const int grid = static_cast<int>((n + per - 1) / per);
  launch_pdl(kino::gemv_kernel, dim3(grid), dim3(kino::GEMV_THREADS), smem, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
      static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), ldy,
      static_cast<int>(batch), static_cast<int>(n), static_cast<int>(k), act);
  return check_launch("kino_gemv");
}

int64_t kino_attention_workspace_size(const kino_attention_args* a, int64_t kv_splits) {
  if (a == nullptr || kv_splits < 1 || a->n_q < 1 || a->n_q > 2 || a->batch < 1 || a->heads < 1)
    return -1;
  if (kv_splits == 1) return 0;
  int64_t tiles = 0;
  for (int s = 0; s < a->n_q; ++s) tiles += (a->q_tokens[s] + 127) / 128;
  const int64_t rows = (tiles + 1) / 2 * 2 * 128;
  const int64_t n = kv_splits * a->batch * a->heads * rows;
  return n * a->head_dim * 4 + n * 2 * 4;
}

kino_status kino_attention(const kino_attention_args* a, void* stream) {
  if (a == nullptr) return fail(KINO_EINVAL, "kino_attention: null args");
  if (a->head_dim != 128 && a->head_dim != 64)
    return fail(KINO_ENOTSUPPORTED, "kino_attention: head_dim %lld (64 or 128)",
                (long long)a->head_dim);
  const uint64_t hd = static_cast<uint64_t>(a->head_dim);
  if (a->n_q < 1 || a->n_q > 2 || a->n_kv < 1 || a->n_kv > 2)
    return fail(KINO_EINVAL, "kino_attention: 1 or 2 segments");
  if (a->batch < 1 || a->heads < 1 || a->batch > 65535 || a->heads > 65535)
    return fail(KINO_EINVAL, "kino_attention: batch/heads");
  kino::AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.batch = static_cast<int>(a->batch);
  p.heads = static_cast<int>(a->heads);
  p.nq_seg = a->n_q;
  p.nkv_seg = a->n_kv;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  CUtensorMap mq[2], mk[2], mv[2];
  const uint32_t box[4] = {64, kino::ATT_BM, 1, 1};
  const uint32_t kvbox[4] = {64, kino::ATT_BN, 1, 1};
  int tiles = 0;
  for (int s = 0; s < 2; ++s) {
    const int qs = s < a->n_q ? s : 0;
    if (s < a->n_q && (a->q_tokens[s] < 1 || a->q[s] == nullptr || a->out[s] == nullptr))
      return fail(KINO_EINVAL, "kino_attention: empty query segment");
    if (a->ld_q[qs] % 8 || a->ld_out[qs] % 8 || (a->batch > 1 && (a->bs_q[qs] % 8)))
      return fail(KINO_ENOTSUPPORTED, "kino_attention: strides must be multiples of 8");
    const uint64_t dq[4] = {hd, static_cast<uint64_t>(a->q_tokens[qs]),
                            static_cast<uint64_t>(a->heads), static_cast<uint64_t>(a->batch)};
    const uint64_t sq[3] = {static_cast<uint64_t>(a->ld_q[qs]), hd,
                            static_cast<uint64_t>(a->batch > 1 ? a->bs_q[qs] : 8)};
    kino_status st = make_map(&mq[s], a->q[qs], 4, dq, sq, box);
    if (st != KINO_OK) return st;
    if (!aligned16(a->out[qs])) return fail(KINO_EINVAL, "kino_attention: out alignment");
    if (s < a->n_q) {
      p.q_tokens[s] = static_cast<int>(a->q_tokens[s]);
      p.q_tiles[s] = (p.q_tokens[s] + 127) / 128;
      p.out[s] = static_cast<__nv_bfloat16*>(a->out[s]);
      p.ld_out[s] = a->ld_out[s];
      p.bs_out[s] = a->bs_out[s];
      p.gate[s] = static_cast<const __nv_bfloat16*>(a->gate[s]);
      p.ld_gate[s] = a->ld_gate[s];
      p.bs_gate[s] = a->bs_gate[s];
      tiles += p.q_tiles[s];
    }
    const int ks = s < a->n_kv ? s : 0;
    if (s < a->n_kv && (a->kv_tokens[s] < 1 || a->k[s] == nullptr || a->v[s] == nullptr))
      return fail(KINO_EINVAL, "kino_attention: empty key segment");
    if (a->ld_k[ks] % 8 || a->ld_v[ks] % 8 ||
        (a->batch > 1 && (a->bs_k[ks] % 8 || a->bs_v[ks] % 8)))
      return fail(KINO_ENOTSUPPORTED, "kino_attention: strides must be multiples of 8");
    const uint64_t dk[4] = {hd, static_cast<uint64_t>(a->kv_tokens[ks]),
                            static_cast<uint64_t>(a->heads), static_cast<uint64_t>(a->batch)};
    const uint64_t sk[3] = {static_cast<uint64_t>(a->ld_k[ks]), hd,
                            static_cast<uint64_t>(a->batch > 1 ? a->bs_k[ks] : 8)};
    const uint64_t sv[3] = {static_cast<uint64_t>(a->ld_v[ks]), hd,
                            static_cast<uint64_t>(a->batch > 1 ? a->bs_v[ks] : 8)};
    st = make_map(&mk[s], a->k[ks], 4, dk, sk, kvbox);
    if (st != KINO_OK) return st;
    st = make_map(&mv[s], a->v[ks], 4, dk, sv, kvbox);
    if (st != KINO_OK) return st;
    if (s < a->n_kv) {
      p.kv_tokens[s] = static_cast<int>(a->kv_tokens[s]);
      p.kv_blocks[s] = (p.kv_tokens[s] + kino::ATT_BN - 1) / kino::ATT_BN;
    }
  }
  if (a->out_peers != nullptr) {
    if (a->batch != 1 || a->n_q != 1)
      return fail(KINO_EINVAL, "kino_attention: peer return needs batch 1, one query segment");
    if (a->world < 1 || a->world > kino::PEER_MAX_WORLD || a->rows_per_rank < 1 ||
        a->rows_per_rank * a->world < a->q_tokens[0] || a->out_col_offset < 0 ||
        a->out_col_offset % 8 || a->out_col_offset + a->heads * a->head_dim > a->out_cols ||
        a->out_cols > a->ld_out[0])
      return fail(KINO_EINVAL, "kino_attention: peer return rows/columns outside the buffers");
    if (a->gate_peers != nullptr &&
        (a->gate_head_offset < 0 || a->gate_head_offset + a->heads > a->ld_gate[0]))
      return fail(KINO_EINVAL, "kino_attention: peer gate columns outside the gate rows");
    p.out_peers = reinterpret_cast<__nv_bfloat16* const*>(a->out_peers);
    p.gate_peers = reinterpret_cast<const __nv_bfloat16* const*>(a->gate_peers);
    p.rows_per_rank = static_cast<int>(a->rows_per_rank);
    p.out_col_offset = a->out_col_offset;
    p.gate_head_offset = static_cast<int>(a->gate_head_offset);
    p.ld_out[0] = a->ld_out[0];
    p.ld_gate[0] = a->ld_gate[0];
  }
  const int splits = a->kv_splits > 1 ? static_cast<int>(a->kv_splits) : 1;
  if (splits > 1) {
    const int nblk_all = p.kv_blocks[0] + (a->n_kv > 1 ? p.kv_blocks[1] : 0);
    if (a->key_bias != nullptr)
      return fail(KINO_EINVAL, "kino_attention: a key bias takes no key split");
    if (splits > nblk_all || splits > 16)
      return fail(KINO_EINVAL, "kino_attention: kv_splits %d outside 1 .. min(16, %d key blocks)",
                  splits, nblk_all);
    const int64_t need = kino_attention_workspace_size(a, splits);
    if (a->workspace == nullptr || a->workspace_bytes < need || !aligned16(a->workspace))
      return fail(KINO_EINVAL, "kino_attention: a %d-way key split needs %lld bytes of 16-byte "
                  "aligned workspace", splits, (long long)need);
    p.kv_splits = splits;
    p.part_rows = static_cast<int64_t>((tiles + 1) / 2) * 2 * kino::ATT_BM;
    p.part_o = static_cast<float*>(a->workspace);
    p.part_ml = p.part_o + static_cast<int64_t>(splits) * p.batch * p.heads * p.part_rows * hd;
  }
  // two 128-query tiles per CTA, each CTA on one share of the keys when they are split
  dim3 grid(static_cast<unsigned>((tiles + 1) / 2 * splits), p.heads, p.batch);
  auto run = [&](auto kernel, int slot) {
    kino_status st = ensure_smem(kernel, kino::AttnSmem::TOTAL, slot);
    if (st != KINO_OK) return st;
    launch_pdl(kernel, dim3(grid), dim3(kino::ATT_THREADS), kino::AttnSmem::TOTAL,
               static_cast<cudaStream_t>(stream), mq[0], mq[1], mk[0], mk[1], mv[0], mv[1], p);
    st = check_launch("kino_attention");
    if (st != KINO_OK || splits == 1) return st;
    const int64_t threads = static_cast<int64_t>(p.batch) * p.heads * p.part_rows * (hd / 8);
    const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
    if (hd == 64)
      launch_pdl(kino::attention_combine_kernel<64>, dim3(blocks), dim3(256), 0,
                 static_cast<cudaStream_t>(stream), p);
    else
      launch_pdl(kino::attention_combine_kernel<128>, dim3(blocks), dim3(256), 0,
                 static_cast<cudaStream_t>(stream), p);
    return check_launch("kino_attention (combine)");
  };
  if (a->key_bias != nullptr) {
    if (a->n_kv != 1 || a->out_peers != nullptr)
      return fail(KINO_EINVAL, "kino_attention: a key bias takes one key segment, no peer return");
    const int64_t padded = (a->kv_tokens[0] + 3) / 4 * 4;
    if (!aligned16(a->key_bias) || a->ld_key_bias % 4 ||
        (a->batch > 1 && a->ld_key_bias < padded))
      return fail(KINO_EINVAL,
                  "kino_attention: key bias rows 16-byte aligned, stride a multiple of 4 floats "
                  "covering the keys rounded up to 4");
    p.key_bias = a->key_bias;
    p.ld_key_bias = a->ld_key_bias;
    return a->head_dim == 64 ? run(kino::attention_tc_kernel<64, true>, 14)
                             : run(kino::attention_tc_kernel<128, true>, 15);
  }
  if (splits > 1)
    return a->head_dim == 64 ? run(kino::attention_tc_kernel<64, false, true>, 27)
                             : run(kino::attention_tc_kernel<128, false, true>, 28);
  return a->head_dim == 64 ? run(kino::attention_tc_kernel<64>, 11)
                           : run(kino::attention_tc_kernel<128>, 3);
}

// ---------------------------------------------------------------- Sol-Attn
int64_t kino_sol_attention_workspace_size(int64_t tokens, int64_t heads) {
  if (tokens < 1 || heads < 1 || tokens > (int64_t{1} << 30) || heads > 256) {
    fail(KINO_EINVAL, "kino_sol_attention_workspace_size: tokens/heads");
    return -1;
  }
  return sol_layout(tokens, heads).total;
}

kino_status kino_sol_attention(const kino_sol_attention_args* a, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr ||
      a->out == nullptr || a->order == nullptr || a->workspace == nullptr)
    return fail(KINO_EINVAL, "kino_sol_attention: null argument");
  if (a->tokens < 1 || a->heads < 1 || a->heads > 256)
    return fail(KINO_EINVAL, "kino_sol_attention: tokens/heads");
  if (a->dtype != KINO_DTYPE_BF16 && a->dtype != KINO_DTYPE_F16)
    return fail(KINO_EINVAL, "kino_sol_attention: dtype must be KINO_DTYPE_BF16 or KINO_DTYPE_F16");
  if (!(a->tau == a->tau) || a->tau > 3.0e38f || a->tau < -3.0e38f)
    return fail(KINO_EINVAL, "kino_sol_attention: tau must be finite");
  const SolLayout l = sol_layout(a->tokens, a->heads);
  if (l.nb > kino::SOL_MAX_WORDS * 32)
    return fail(KINO_ENOTSUPPORTED, "kino_sol_attention: at most %d blocks of 64 tokens",
                kino::SOL_MAX_WORDS * 32);
  if (a->workspace_bytes < l.total || !aligned16(a->workspace))
    return fail(KINO_EINVAL, "kino_sol_attention: workspace below %lld bytes or unaligned",
                (long long)l.total);
  if (a->ld_q < l.width || a->ld_k < l.width || a->ld_v < l.width || a->ld_out < l.width ||
      a->ld_q % 8 || a->ld_k % 8 || a->ld_v % 8 || a->ld_out % 8 || !aligned16(a->q) ||
      !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
    return fail(KINO_ENOTSUPPORTED,
                "kino_sol_attention: row strides >= heads * 128, multiples of 8, aligned rows");
  if (a->gate != nullptr && a->ld_gate < a->heads)
    return fail(KINO_EINVAL, "kino_sol_attention: gate stride below heads");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  __half* q16 = reinterpret_cast<__half*>(ws + l.q16);
  __half* k16 = reinterpret_cast<__half*>(ws + l.k16);
  __half* v16 = reinterpret_cast<__half*>(ws + l.v16);
  float* qmean = reinterpret_cast<float*>(ws + l.qmean);
  __half* kmean = reinterpret_cast<__half*>(ws + l.kmean);
  __half* vmean = reinterpret_cast<__half*>(ws + l.vmean);
  uint32_t* bits = a->routes != nullptr ? a->routes : reinterpret_cast<uint32_t*>(ws + l.bits);
  int* lists = reinterpret_cast<int*>(ws + l.lists);
  int* counts = reinterpret_cast<int*>(ws + l.counts);
  const int tokens = static_cast<int>(a->tokens), heads = static_cast<int>(a->heads);
  const dim3 grid_bh(static_cast<unsigned>(l.nb), static_cast<unsigned>(heads));
  if (a->dtype == KINO_DTYPE_F16)
    launch_pdl(kino::sol_prepare_kernel<__half>, grid_bh, dim3(128), 0, st,
               static_cast<const __half*>(a->q), static_cast<const __half*>(a->k),
               static_cast<const __half*>(a->v), a->ld_q, a->ld_k, a->ld_v, a->order, tokens,
               heads, q16, k16, v16, qmean, kmean, vmean);
  else
    launch_pdl(kino::sol_prepare_kernel<__nv_bfloat16>, grid_bh, dim3(128), 0, st,
               static_cast<const __nv_bfloat16*>(a->q), static_cast<const __nv_bfloat16*>(a->k),
               static_cast<const __nv_bfloat16*>(a->v), a->ld_q, a->ld_k, a->ld_v, a->order,
               tokens, heads, q16, k16, v16, qmean, kmean, vmean);
  kino_status s = check_launch("kino_sol_attention (prepare)");
  if (s != KINO_OK) return s;
  const double ls = 1.4426950408889634 / sqrt(128.0);
  const dim3 grid_route(static_cast<unsigned>((l.nb + kino::SOL_ROUTE_ROWS - 1) / kino::SOL_ROUTE_ROWS),
                        static_cast<unsigned>(heads));
  const int route_smem = kino::sol_route_smem(static_cast<int>(l.nb));
  if ((s = ensure_smem(kino::sol_route_kernel, kino::sol_route_smem(kino::SOL_MAX_WORDS * 32), 13)) !=
      KINO_OK)
    return s;
  launch_pdl(kino::sol_route_kernel, grid_route, dim3(256), route_smem, st, qmean, kmean,
             static_cast<int>(l.nb), static_cast<int>(l.words), static_cast<float>(ls),
             static_cast<float>(ls * ls), a->tau, bits);
  s = check_launch("kino_sol_attention (route)");
  if (s != KINO_OK) return s;
  launch_pdl(kino::sol_union_kernel, dim3(static_cast<unsigned>(l.ncta), heads), dim3(32), 0, st,
             bits, static_cast<int>(l.nb), static_cast<int>(l.words), lists, counts);
  s = check_launch("kino_sol_attention (union)");
  if (s != KINO_OK) return s;
  CUtensorMap mq, mk, mv, mkc, mvc;
  const uint64_t dq[4] = {128, static_cast<uint64_t>(tokens), static_cast<uint64_t>(heads), 1};
  const uint64_t sq[3] = {static_cast<uint64_t>(l.width), 128, 8};
  const uint32_t qbox[4] = {64, 128, 1, 1};
  const uint32_t kbox[4] = {64, 64, 1, 1};
  if ((s = make_map(&mq, q16, 4, dq, sq, qbox)) != KINO_OK) return s;
  if ((s = make_map(&mk, k16, 4, dq, sq, kbox)) != KINO_OK) return s;
  if ((s = make_map(&mv, v16, 4, dq, sq, kbox)) != KINO_OK) return s;
  const uint64_t dc[3] = {128, static_cast<uint64_t>(l.nb), static_cast<uint64_t>(heads)};
  const uint64_t sc[2] = {128, static_cast<uint64_t>(l.nb * 128)};
  const uint32_t cbox[3] = {64, 64, 1};
  if ((s = make_map(&mkc, kmean, 3, dc, sc, cbox)) != KINO_OK) return s;
  if ((s = make_map(&mvc, vmean, 3, dc, sc, cbox)) != KINO_OK) return s;
  kino::SolParams p;
  std::memset(&p, 0, sizeof(p));
  p.tokens = tokens;
  p.heads = heads;
  p.nb = static_cast<int>(l.nb);
  p.words = static_cast<int>(l.words);
  p.ncta = static_cast<int>(l.ncta);
  p.scale_log2 = static_cast<float>(ls);
  p.last_log2 = static_cast<float>(log2(static_cast<double>(tokens - (l.nb - 1) * kino::SOL_BLOCK)));
  p.bits = bits;
  p.lists = lists;
  p.counts = counts;
  p.order = a->order;
  p.out = a->out;
  p.ld_out = a->ld_out;
  p.out_f16 = a->dtype == KINO_DTYPE_F16 ? 1 : 0;
  p.gate = a->gate;
  p.ld_gate = a->ld_gate;
  constexpr int smem = kino::SolSmem::TOTAL;
  if ((s = ensure_smem(kino::sol_attention_kernel, smem, 12)) != KINO_OK) return s;
  const int64_t items = l.ncta * heads;  // (head, query tile) work items, one CTA per SM
  const unsigned persistent = static_cast<unsigned>(std::min<int64_t>(items, device_sms()));
  launch_pdl(kino::sol_attention_kernel, dim3(persistent),
             dim3(kino::ATT_THREADS), smem, st, mq, mk, mv, mkc, mvc, p);
  return check_launch("kino_sol_attention");
}

kino_status kino_neighborhood_attention(const void* q, const void* k, const void* v, void* out,
                                        int64_t batch, int64_t frames, int64_t height,
                                        int64_t width, int64_t heads, const int32_t* window,
                                        void* stream) {
  return kino_neighborhood_attention_ex(q, k, v, out, KINO_DTYPE_F16, batch, frames, height, width,
                                        heads, window, stream);
}

kino_status kino_neighborhood_attention_ex(const void* q, const void* k, const void* v, void* out,
                                           int out_dtype, int64_t batch, int64_t frames,
                                           int64_t height, int64_t width, int64_t heads,
                                           const int32_t* window, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || window == nullptr)
    return fail(KINO_EINVAL, "kino_neighborhood_attention: null argument");
  if (out_dtype != KINO_DTYPE_F16 && out_dtype != KINO_DTYPE_BF16)
    return fail(KINO_EINVAL, "kino_neighborhood_attention: out_dtype is KINO_DTYPE_F16 or _BF16");
  if (batch < 1 || frames < 1 || height < 1 || width < 1 || heads < 1 || heads > 4096 ||
      batch * frames > 0x7fffffff || height > 0x7fffffff || width > 0x7fffffff)
    return fail(KINO_EINVAL, "kino_neighborhood_attention: empty or oversized grid");
  const int64_t ext[3] = {frames, height, width};
  for (int a = 0; a < 3; ++a)
    if (window[a] < 1 || window[a] % 2 == 0 || window[a] > ext[a])
      return fail(KINO_EINVAL, "kino_neighborhood_attention: window %d on axis %d must be odd "
                  "and no larger than the grid (%lld)", window[a], a, (long long)ext[a]);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(KINO_EINVAL, "kino_neighborhood_attention: operands must be 16-byte aligned");
  kino::NaParams p;
  std::memset(&p, 0, sizeof(p));
  p.batch = static_cast<int>(batch);
  p.frames = static_cast<int>(frames);
  p.height = static_cast<int>(height);
  p.width = static_cast<int>(width);
  p.heads = static_cast<int>(heads);
  p.kt = window[0];
  p.kh = window[1];
  p.kw = window[2];
  p.boxes_t = static_cast<int>((frames + kino::NA_QT - 1) / kino::NA_QT);
  p.boxes_h = static_cast<int>((height + kino::NA_QH - 1) / kino::NA_QH);
  p.boxes_w = static_cast<int>((width + kino::NA_QW - 1) / kino::NA_QW);
  p.scale_log2 = 1.4426950408889634f;  // the queries arrive scaled: softmax(q k^T)
  p.out = static_cast<__half*>(out);
  p.out_bf16 = out_dtype == KINO_DTYPE_BF16 ? 1 : 0;
  const int64_t items = batch * heads * p.boxes_t * p.boxes_h * p.boxes_w;
  if (items > 0x7fffffff)
    return fail(KINO_ENOTSUPPORTED, "kino_neighborhood_attention: too many query tiles");
  // (head dim, head, width, height, batch * frames), strides in elements
  const uint64_t dims[5] = {64, static_cast<uint64_t>(heads), static_cast<uint64_t>(width),
                            static_cast<uint64_t>(height), static_cast<uint64_t>(batch * frames)};
  const uint64_t strides[4] = {64, static_cast<uint64_t>(heads * 64),
                               static_cast<uint64_t>(width * heads * 64),
                               static_cast<uint64_t>(height * width * heads * 64)};
  const uint32_t qbox[5] = {64, 1, kino::NA_QW, kino::NA_QH, kino::NA_TILE_T};  // one tile
  const uint32_t kbox[5] = {64, 1, kino::NA_KW, kino::NA_KH, 1};
  CUtensorMap mq, mk, mv;
  kino_status s;
  if ((s = make_map(&mq, q, 5, dims, strides, qbox)) != KINO_OK) return s;
  if ((s = make_map(&mk, k, 5, dims, strides, kbox)) != KINO_OK) return s;
  if ((s = make_map(&mv, v, 5, dims, strides, kbox)) != KINO_OK) return s;
  constexpr int smem = kino::NaSmem::TOTAL;
  if ((s = ensure_smem(kino::na_attention_kernel, smem, 22)) != KINO_OK) return s;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, device_sms()));
  launch_pdl(kino::na_attention_kernel, dim3(grid), dim3(kino::ATT_THREADS), smem,
             static_cast<cudaStream_t>(stream), mq, mk, mv, p);
  return check_launch("kino_neighborhood_attention");
}

kino_status kino_na_qkv_prepare(const void* qkv, int64_t ld, void* q, void* k, void* v,
                                const void* q_norm_weight, const void* k_norm_weight,
                                const float* rope_tables, int64_t batch, int64_t frames,
                                int64_t height, int64_t width, int64_t heads,
                                const int32_t* section_pairs, float q_scale, float eps,
                                void* stream) {
  if (qkv == nullptr || q == nullptr || k == nullptr || v == nullptr ||
      q_norm_weight == nullptr || k_norm_weight == nullptr || rope_tables == nullptr ||
      section_pairs == nullptr)
    return fail(KINO_EINVAL, "kino_na_qkv_prepare: null operand");
  if (batch < 1 || frames < 1 || height < 1 || width < 1 || heads < 1 || heads > 1024)
    return fail(KINO_EINVAL, "kino_na_qkv_prepare: empty or oversized shape");
  const int64_t tokens = batch * frames * height * width;
  if (tokens > (int64_t(1) << 31) || ld < 3 * heads * 64 || ld % 8)
    return fail(KINO_EINVAL, "kino_na_qkv_prepare: row stride below 3 * heads * 64 or unaligned");
  const int pt = section_pairs[0], ph = section_pairs[1], pw = section_pairs[2];
  if (pt < 0 || ph < 0 || pw < 0 || pt + ph + pw != 32)
    return fail(KINO_EINVAL, "kino_na_qkv_prepare: the t, h, w sections must hold 32 pairs");
  if (!aligned16(qkv) || !aligned16(v) || !aligned16(q) || !aligned16(k) ||
      !aligned16(q_norm_weight) || !aligned16(k_norm_weight))
    return fail(KINO_EINVAL, "kino_na_qkv_prepare: operands must be 16-byte aligned");
  kino::NaPrepParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld = ld;
  p.q = static_cast<__half*>(q);
  p.k = static_cast<__half*>(k);
  p.v = static_cast<__half*>(v);
  p.wq = static_cast<const __nv_bfloat16*>(q_norm_weight);
  p.wk = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.tables = rope_tables;
  p.tokens = tokens;
  p.heads = static_cast<int>(heads);
  p.gt = static_cast<int>(frames);
  p.gh = static_cast<int>(height);
  p.gw = static_cast<int>(width);
  p.pt = pt;
  p.ph = ph;
  p.pw = pw;
  p.q_scale = q_scale;
  p.eps = eps;
  const int64_t blocks = (tokens + kino::NAP_THREADS / 32 - 1) / (kino::NAP_THREADS / 32);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks, 32LL * device_sms()));
  launch_pdl(kino::na_qkv_prepare_kernel, dim3(grid), dim3(kino::NAP_THREADS), 0,
             static_cast<cudaStream_t>(stream), p);
  return check_launch("kino_na_qkv_prepare");
}

kino_status kino_strided_copy(const void* src, int src_dtype, const int64_t* src_strides,
                              void* dst, int dst_dtype, const int64_t* dst_strides,
                              const int64_t* sizes, int ndim, void* stream) {
  if (src == nullptr || dst == nullptr || src_strides == nullptr || dst_strides == nullptr ||
      sizes == nullptr)
    return fail(KINO_EINVAL, "kino_strided_copy: null operand");
  if (ndim < 1 || ndim > kino::COPY_MAX_DIMS)
    return fail(KINO_EINVAL, "kino_strided_copy: 1..%d dimensions", kino::COPY_MAX_DIMS);
  if (src_dtype < KINO_DTYPE_BF16 || src_dtype > KINO_DTYPE_F32 || dst_dtype < KINO_DTYPE_BF16 ||
      dst_dtype > KINO_DTYPE_F32)
    return fail(KINO_EINVAL, "kino_strided_copy: dtypes are KINO_DTYPE_BF16, _F16 or _F32");
  kino::CopyParams p;
  std::memset(&p, 0, sizeof(p));
  p.src = src;
  p.dst = dst;
  p.ndim = ndim;
  p.src_type = src_dtype;
  p.dst_type = dst_dtype;
  int64_t total = 1;
  int64_t largest = 1;
  for (int d = 0; d < kino::COPY_MAX_DIMS; ++d) p.size[d] = 1;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] < 0) return fail(KINO_EINVAL, "kino_strided_copy: negative size");
    if (dst_strides[d] < 0) return fail(KINO_EINVAL, "kino_strided_copy: negative destination stride");
    p.size[d] = sizes[d];
    p.src_stride[d] = src_strides[d];
    p.dst_stride[d] = dst_strides[d];
    total *= sizes[d];
    largest = std::max(largest, sizes[d]);
  }
  if (total == 0) return KINO_OK;
  p.total = total;
  const bool vec = sizes[ndim - 1] % 8 == 0;
  const int64_t blocks = (total / (vec ? 8 : 1) + kino::COPY_THREADS - 1) / kino::COPY_THREADS;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks, 16LL * device_sms()));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool narrow = total <= 0xffffffffLL && largest <= 0xffffffffLL;
  const dim3 g(grid), b(kino::COPY_THREADS);
  if (narrow && vec)
    launch_pdl(kino::strided_copy_kernel<uint32_t, 8>, g, b, 0, st, p);
  else if (narrow)
    launch_pdl(kino::strided_copy_kernel<uint32_t, 1>, g, b, 0, st, p);
  else if (vec)
    launch_pdl(kino::strided_copy_kernel<uint64_t, 8>, g, b, 0, st, p);
  else
    launch_pdl(kino::strided_copy_kernel<uint64_t, 1>, g, b, 0, st, p);
  return check_launch("kino_strided_copy");
}

kino_status kino_dense_attention(const void* q, const void* k, const void* v, void* out,
                                 int64_t tq, int64_t tk, int64_t heads, int64_t dim,
                                 void* stream) {
  if (dim != 128 && dim != 64)
    return fail(KINO_ENOTSUPPORTED, "kino_dense_attention: dim %lld (64 or 128)", (long long)dim);
  kino_attention_args a;
  std::memset(&a, 0, sizeof(a));
  a.batch = 1;
  a.heads = heads;
  a.head_dim = dim;
  a.scale = 1.0f / sqrtf(static_cast<float>(dim));
  a.n_q = 1;
  a.q[0] = q;
  a.out[0] = out;
  a.q_tokens[0] = tq;
  a.ld_q[0] = a.ld_out[0] = heads * dim;
  a.n_kv = 1;
  a.k[0] = k;
  a.v[0] = v;
  a.kv_tokens[0] = tk;
  a.ld_k[0] = a.ld_v[0] = heads * dim;
  return kino_attention(&a, stream);
}

kino_status kino_adaln(const void* x, int64_t ldx, int64_t bsx, const void* shift,
                       const void* scale, int64_t bs_mod, void* out, int64_t ldo, int64_t bso,
                       int64_t batch, int64_t rows, int64_t dim, int norm_kind, float eps,
                       void* stream) {
  if (x == nullptr || shift == nullptr || scale == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_adaln: null");
  if (dim % 8 || dim > 8192 || ldx % 8 || ldo % 8 || bs_mod % 8 || !aligned16(x) ||
      !aligned16(out) || !aligned16(shift) || !aligned16(scale))
    return fail(KINO_ENOTSUPPORTED, "kino_adaln: dim %% 8, dim <= 8192, aligned operands");
  if (rows < 1 || batch < 1 || rows > 0x7fffffff || batch > 65535)
    return fail(KINO_EINVAL, "kino_adaln: rows/batch");
  if (norm_kind < 0 || norm_kind > 2) return fail(KINO_EINVAL, "kino_adaln: norm kind");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // warp per row where the width is a multiple of 256 the kernel is instantiated for: a
  // grid-stride kernel with as many CTAs as fit on the SMs at once (two row slots per warp in
  // shared memory), or fewer when the rows run out
  auto warp_form = [&](auto kernel, int vpl, int slot) {
    const int smem = kino::adaln_stream_smem(vpl);
    kino_status s = ensure_smem(kernel, smem, slot);
    if (s != KINO_OK) return s;
    const int static_bytes = vpl * 256 * 4;  // shift and bf16(1 + scale)
    const int per_sm = std::max(1, std::min(4, (227 * 1024) / (smem + static_bytes + 1024)));
    const int64_t need = (rows + kino::ADALN_WARPS - 1) / kino::ADALN_WARPS;
    const int64_t fit = std::max<int64_t>(1, int64_t{per_sm} * device_sms() / batch);
    dim3 wgrid(static_cast<unsigned>(std::min(need, fit)), static_cast<unsigned>(batch));
    launch_pdl(kernel, dim3(wgrid), dim3(kino::ADALN_WARPS * 32), smem, st,
        static_cast<const __nv_bfloat16*>(x), ldx, bsx, static_cast<const __nv_bfloat16*>(shift),
        static_cast<const __nv_bfloat16*>(scale), bs_mod, static_cast<__nv_bfloat16*>(out), ldo,
        bso, static_cast<int>(rows), norm_kind, eps);
    return check_launch("kino_adaln");
  };
  switch (dim) {
    case 256: return warp_form(kino::adaln_warp_kernel<1>, 1, 16);
    case 512: return warp_form(kino::adaln_warp_kernel<2>, 2, 17);
    case 1024: return warp_form(kino::adaln_warp_kernel<4>, 4, 18);
    case 2048: return warp_form(kino::adaln_warp_kernel<8>, 8, 19);
    case 3072: return warp_form(kino::adaln_warp_kernel<12>, 12, 20);
    case 4096: return warp_form(kino::adaln_warp_kernel<16>, 16, 21);
    default: break;
  }
  dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(batch));
  launch_pdl(kino::adaln_kernel, dim3(grid), dim3(kino::ADALN_THREADS), 0, st,
      static_cast<const __nv_bfloat16*>(x), ldx, bsx, static_cast<const __nv_bfloat16*>(shift),
      static_cast<const __nv_bfloat16*>(scale), bs_mod, static_cast<__nv_bfloat16*>(out), ldo,
      bso, static_cast<int>(rows), static_cast<int>(dim), norm_kind, eps);
  return check_launch("kino_adaln");
}

kino_status kino_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t dim,
                          float eps, float weight_offset, void* stream) {
  if (x == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_rms_norm: null");
  if (dim % 8 || dim > 8192 || !aligned16(x) || !aligned16(out) ||
      (weight != nullptr && !aligned16(weight)))
    return fail(KINO_ENOTSUPPORTED, "kino_rms_norm: dim %% 8, dim <= 8192, aligned operands");
  if (rows < 1 || rows > 0x7fffffff) return fail(KINO_EINVAL, "kino_rms_norm: rows");
  if (dim <= 1024) {  // a warp per row
    const int64_t blocks = (rows + kino::RMS_WARP_THREADS / 32 - 1) / (kino::RMS_WARP_THREADS / 32);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks, 16LL * device_sms()));
    auto run = [&](auto kernel) {
      launch_pdl(kernel, dim3(grid), dim3(kino::RMS_WARP_THREADS), 0,
                 static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                 static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), rows,
                 static_cast<int>(dim), eps, weight_offset);
    };
    if (dim <= 256)
      run(kino::rms_norm_warp_kernel<1>);
    else if (dim <= 512)
      run(kino::rms_norm_warp_kernel<2>);
    else
      run(kino::rms_norm_warp_kernel<4>);
    return check_launch("kino_rms_norm");
  }
  launch_pdl(kino::rms_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kino::ADALN_THREADS), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
      static_cast<__nv_bfloat16*>(out), static_cast<int>(dim), eps, weight_offset);
  return check_launch("kino_rms_norm");
}

kino_status kino_qk_norm_rope(void* x, int64_t ld, int64_t bs, int64_t batch, int64_t tokens,
                              int64_t heads, const void* weight, int norm_kind, int rope_kind,
                              const float* cos_table, const float* sin_table, int table_batched,
                              int64_t table_tokens, int64_t table_offset, float eps,
                              void* stream) {
  if (x == nullptr) return fail(KINO_EINVAL, "kino_qk_norm_rope: null");
  if (norm_kind < 0 || norm_kind > 2 || rope_kind < 0 || rope_kind > 3)
    return fail(KINO_EINVAL, "kino_qk_norm_rope: bad kind");
  if (rope_kind == 3 && norm_kind == 1)
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope: 64-wide heads take the full-row norm");
  if (norm_kind != 0 && (weight == nullptr || !aligned16(weight)))
    return fail(KINO_EINVAL, "kino_qk_norm_rope: norm needs an aligned weight");
  if (rope_kind != 0 && (cos_table == nullptr || sin_table == nullptr))
    return fail(KINO_EINVAL, "kino_qk_norm_rope: rope needs tables");
  if (heads < 1 || heads > 128 || ld % 8 || (batch > 1 && bs % 8) || !aligned16(x))
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope: heads <= 128, aligned rows");
  if (tokens < 1 || batch < 1) return fail(KINO_EINVAL, "kino_qk_norm_rope: empty");
  if (rope_kind != 0 && table_offset + tokens > table_tokens)
    return fail(KINO_EINVAL, "kino_qk_norm_rope: table too short");
  dim3 grid(static_cast<unsigned>(tokens), static_cast<unsigned>(batch));
  launch_pdl(kino::qk_norm_rope_kernel, dim3(grid), dim3(static_cast<unsigned>(heads * 8)), 0, static_cast<cudaStream_t>(stream),
      static_cast<__nv_bfloat16*>(x), ld, bs, static_cast<int>(heads),
      static_cast<const __nv_bfloat16*>(weight), norm_kind, rope_kind, cos_table, sin_table,
      table_batched, static_cast<int>(table_tokens), static_cast<int>(table_offset), eps,
      static_cast<__nv_bfloat16* const*>(nullptr), 0, int64_t{0}, int64_t{0}, 0);
  return check_launch("kino_qk_norm_rope");
}

kino_status kino_qk_norm_rope_to_peers(const void* x, int64_t ld, int64_t tokens, int64_t heads,
                                       const void* weight, int norm_kind, int rope_kind,
                                       const float* cos_table, const float* sin_table,
                                       int table_batched, int64_t table_tokens,
                                       int64_t table_offset, float eps, void* const* dst_ptrs,
                                       int64_t world, int64_t dst_ld, int64_t dst_row0,
                                       int64_t dst_rows, int64_t dst_slot, void* stream) {
  if (x == nullptr || dst_ptrs == nullptr) return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: null");
  if (norm_kind < 0 || norm_kind > 2 || rope_kind < 0 || rope_kind > 2)
    return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: bad kind");
  if (norm_kind != 0 && (weight == nullptr || !aligned16(weight)))
    return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: norm needs an aligned weight");
  if (rope_kind != 0 && (cos_table == nullptr || sin_table == nullptr))
    return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: rope needs tables");
  if (heads < 1 || heads > 128 || ld % 8 || !aligned16(x))
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_to_peers: heads <= 128, aligned rows");
  if (tokens < 1) return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: empty");
  if (rope_kind != 0 && table_offset + tokens > table_tokens)
    return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: table too short");
  if (world < 1 || world > kino::PEER_MAX_WORLD || heads % world || dst_ld % 8 || dst_row0 < 0 ||
      dst_row0 + tokens > dst_rows || dst_slot < 0 || (dst_slot + 1) * (heads / world) * 128 > dst_ld)
    return fail(KINO_EINVAL, "kino_qk_norm_rope_to_peers: destination outside the receive buffers");
  launch_pdl(kino::qk_norm_rope_kernel, dim3(static_cast<unsigned>(tokens), 1),
             dim3(static_cast<unsigned>(heads * 8)), 0, static_cast<cudaStream_t>(stream),
             const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(x)), ld, int64_t{0},
             static_cast<int>(heads), static_cast<const __nv_bfloat16*>(weight), norm_kind,
             rope_kind, cos_table, sin_table, table_batched, static_cast<int>(table_tokens),
             static_cast<int>(table_offset), eps, reinterpret_cast<__nv_bfloat16* const*>(dst_ptrs),
             static_cast<int>(heads / world), dst_ld, dst_row0, static_cast<int>(dst_slot));
  return check_launch("kino_qk_norm_rope_to_peers");
}

kino_status kino_split_rope(const void* x, const float* cos_table, const float* sin_table,
                            void* out, int64_t batch, int64_t tokens, int64_t heads, int64_t half,
                            int table_batched, void* stream) {
  if (x == nullptr || cos_table == nullptr || sin_table == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_split_rope: null");
  if (batch < 1 || tokens < 1 || heads < 1 || half < 1)
    return fail(KINO_EINVAL, "kino_split_rope: empty");
  const auto aligned = [](const void* p, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
  };
  if (half % 4 == 0 && aligned(x, 8) && aligned(out, 8) && aligned(cos_table, 16) &&
      aligned(sin_table, 16) && batch * tokens <= 0x7fffffffLL && heads * half <= 0x3fffffffLL) {
    const int64_t rows = batch * tokens;
    const unsigned blocks = static_cast<unsigned>(rows < 148 * 16 ? rows : 148 * 16);
    launch_pdl(kino::split_rope_vec4_kernel, dim3(blocks), dim3(256), 0,
               static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x), cos_table,
               sin_table, static_cast<__nv_bfloat16*>(out), static_cast<int>(batch),
               static_cast<int>(tokens), static_cast<int>(heads), static_cast<int>(half),
               table_batched);
    return check_launch("kino_split_rope");
  }
  const int64_t n = batch * tokens * heads * half;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 65535 * 8) blocks = 65535 * 8;
  launch_pdl(kino::split_rope_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(x), cos_table, sin_table,
      static_cast<__nv_bfloat16*>(out), static_cast<int>(batch), static_cast<int>(tokens),
      static_cast<int>(heads), static_cast<int>(half), table_batched);
  return check_launch("kino_split_rope");
}

static kino_status launch_elem(int kind, const void* a, const void* b, void* out, int64_t n,
                               float s0, float s1, void* stream, const char* name) {
  if (a == nullptr || out == nullptr) return fail(KINO_EINVAL, "%s: null", name);
  if (n % 8 || !aligned16(a) || !aligned16(out) || (b != nullptr && !aligned16(b)))
    return fail(KINO_ENOTSUPPORTED, "%s: n %% 8 == 0 and 16-byte alignment required", name);
  if (n == 0) return KINO_OK;
  int64_t blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::elementwise_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      kind, static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
      static_cast<__nv_bfloat16*>(out), n, s0, s1);
  return check_launch(name);
}

kino_status kino_gelu_tanh(const void* x, void* out, int64_t n, void* stream) {
  return launch_elem(kino::ELEM_GELU, x, nullptr, out, n, 0.f, 0.f, stream, "kino_gelu_tanh");
}

kino_status kino_silu(const void* x, void* out, int64_t n, void* stream) {
  return launch_elem(kino::ELEM_SILU, x, nullptr, out, n, 0.f, 0.f, stream, "kino_silu");
}

kino_status kino_cfg_combine(const void* cond, const void* uncond, float guidance, void* out,
                             int64_t n, void* stream) {
  if (uncond == nullptr) return fail(KINO_EINVAL, "kino_cfg_combine: null");
  return launch_elem(kino::ELEM_CFG, cond, uncond, out, n, guidance, 0.f, stream,
                     "kino_cfg_combine");
}

kino_status kino_euler_velocity(const void* x, const void* v, float dt, void* out, int64_t n,
                                void* stream) {
  if (v == nullptr) return fail(KINO_EINVAL, "kino_euler_velocity: null");
  return launch_elem(kino::ELEM_EULER_V, x, v, out, n, dt, 0.f, stream, "kino_euler_velocity");
}

kino_status kino_euler_x0(const void* x, const void* v, float sigma, float ratio, void* out,
                          int64_t n, void* stream) {
  if (v == nullptr) return fail(KINO_EINVAL, "kino_euler_x0: null");
  return launch_elem(kino::ELEM_EULER_X0, x, v, out, n, sigma, ratio, stream, "kino_euler_x0");
}

kino_status kino_euler_step(const void* sample, const void* denoised, float ratio, void* out,
                            int64_t n, void* stream) {
  if (denoised == nullptr) return fail(KINO_EINVAL, "kino_euler_step: null");
  return launch_elem(kino::ELEM_EULER_D, sample, denoised, out, n, 0.f, ratio, stream,
                     "kino_euler_step");
}

kino_status kino_euler_velocity_step(const void* sample, const void* velocity, float delta,
                                     void* out, int64_t n, void* stream) {
  if (velocity == nullptr) return fail(KINO_EINVAL, "kino_euler_velocity_step: null");
  return launch_elem(kino::ELEM_EULER_VS, sample, velocity, out, n, delta, 0.f, stream,
                     "kino_euler_velocity_step");
}

kino_status kino_add_rows(const void* a, const void* b, void* out, int64_t rows, int64_t n,
                          void* stream) {
  if (a == nullptr || b == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_add_rows: null");
  if (n % 8 || !aligned16(a) || !aligned16(b) || !aligned16(out) || rows < 1 || n < 8)
    return fail(KINO_ENOTSUPPORTED, "kino_add_rows: n %% 8 == 0 and aligned operands");
  int64_t blocks = (rows * n / 8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::add_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
      static_cast<__nv_bfloat16*>(out), rows, n);
  return check_launch("kino_add_rows");
}

kino_status kino_heads_pack(const void* src, int64_t ld, void* dst, int64_t tokens,
                           int64_t width, int64_t parts, void* stream) {
  if (src == nullptr || dst == nullptr) return fail(KINO_EINVAL, "kino_heads_pack: null");
  if (parts < 1 || width % (parts * 128) || ld % 8 || !aligned16(src) || !aligned16(dst))
    return fail(KINO_ENOTSUPPORTED, "kino_heads_pack: width must split into 128-wide heads per part");
  int64_t blocks = (tokens * width / 8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) return KINO_OK;
  launch_pdl(kino::heads_pack_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(src), ld, static_cast<__nv_bfloat16*>(dst),
      static_cast<int>(tokens), static_cast<int>(width), static_cast<int>(parts));
  return check_launch("kino_heads_pack");
}

kino_status kino_heads_unpack(const void* src, void* dst, int64_t ld, int64_t tokens,
                             int64_t width, int64_t parts, const void* gate, int64_t ld_gate,
                             void* stream) {
  if (src == nullptr || dst == nullptr) return fail(KINO_EINVAL, "kino_heads_unpack: null");
  if (parts < 1 || width % (parts * 128) || ld % 8 || !aligned16(src) || !aligned16(dst))
    return fail(KINO_ENOTSUPPORTED, "kino_heads_unpack: width must split into 128-wide heads per part");
  int64_t blocks = (tokens * width / 8 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) return KINO_OK;
  launch_pdl(kino::heads_unpack_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), ld,
      static_cast<int>(tokens), static_cast<int>(width), static_cast<int>(parts),
      static_cast<const __nv_bfloat16*>(gate), ld_gate);
  return check_launch("kino_heads_unpack");
}

kino_status kino_timestep_embedding(const float* t, void* out, int64_t batch, int64_t dim,
                                    void* stream) {
  if (t == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_timestep_embedding: null");
  if (batch < 1 || dim < 2 || dim % 2 || batch > 65535)
    return fail(KINO_EINVAL, "kino_timestep_embedding: shape");
  launch_pdl(kino::timestep_embedding_kernel, dim3(static_cast<unsigned>(batch)), dim3(128), 0, static_cast<cudaStream_t>(stream),
      t, static_cast<__nv_bfloat16*>(out), static_cast<int>(batch), static_cast<int>(dim));
  return check_launch("kino_timestep_embedding");
}

#ifndef KINO_CONV_PAIR_BOXES
#define KINO_CONV_PAIR_BOXES 1
#endif
// CTA-pair convolution tiles (M = 256 over two SMs) when enough pair tiles fill the GPU:
// pipeline stages x K blocks per stage (24 KB per block and CTA for 128 output channels,
// 32 KB for 256).
#ifndef KINO_CONV_CTA_PAIRS
#define KINO_CONV_CTA_PAIRS 1
#endif
#ifndef KINO_CONV_HALO
#define KINO_CONV_HALO 1  // CTA-pair convs on W >= 128: one input row per (kt, kh) for three taps
#endif
#ifndef KINO_CONV_NARROW_STAGES
#define KINO_CONV_NARROW_STAGES 2
#endif
#ifndef KINO_CONV_NARROW_KSUB
#define KINO_CONV_NARROW_KSUB 4
#endif
#ifndef KINO_CONV_WIDE_STAGES
#define KINO_CONV_WIDE_STAGES 6
#endif
#ifndef KINO_CONV_WIDE_KSUB
#define KINO_CONV_WIDE_KSUB 1
#endif

kino_status kino_conv3d(const kino_conv3d_args* a, void* stream) {
  if (a == nullptr || a->x == nullptr || a->weight == nullptr || a->out == nullptr)
    return fail(KINO_EINVAL, "kino_conv3d: null operand");
  if (a->frames < 1 || a->height < 1 || a->width < 1 || a->out_channels < 8)
    return fail(KINO_EINVAL, "kino_conv3d: empty shape");
  if (a->in_channels % 64 != 0 || a->in_channels > 8192)
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d: in_channels must be a multiple of 64");
  const int st = a->stride_t, sh = a->stride_h, sw = a->stride_w;
  if (st < 1 || st > 2 || sh < 1 || sh > 2 || sw < 1 || sw > 2)
    return fail(KINO_EINVAL, "kino_conv3d: depth-to-space strides must be 1 or 2");
  const int64_t sub = static_cast<int64_t>(st) * sh * sw;
  if (a->out_channels % sub) return fail(KINO_EINVAL, "kino_conv3d: channels vs strides");
  const int64_t co = a->out_channels / sub;
  if (a->out_channels % 8 || (sub > 1 && co % 32))
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d: output channels per voxel must be 8k (32k with depth-to-space)");
  if (a->residual != nullptr && sub > 1)
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d: residual add only without depth-to-space");
  if (a->workspace != nullptr &&
      (!aligned16(a->workspace) || a->workspace_bytes < KINO_CONV_SPLIT_COUNTERS_BYTES))
    return fail(KINO_EINVAL, "kino_conv3d: workspace must be 16-byte aligned and at least %lld bytes",
                (long long)KINO_CONV_SPLIT_COUNTERS_BYTES);
  if (a->bias != nullptr && !aligned16(a->bias)) return fail(KINO_EINVAL, "kino_conv3d: bias alignment");
  if ((a->residual != nullptr && !aligned16(a->residual)) || !aligned16(a->out))
    return fail(KINO_EINVAL, "kino_conv3d: output/residual alignment");
  if (a->frames * a->height * a->width > (1ll << 31))
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d: too many voxels");
  if (a->stats != nullptr &&
      (co % kino::GN_GROUPS || 32 % (co / kino::GN_GROUPS) || a->out_channels % 32 ||
       !aligned16(a->stats)))
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d: GroupNorm(32) statistics need 32..1024 output "
                                    "channels per voxel with a group size dividing 32");
  kino::ConvShape s;
  std::memset(&s, 0, sizeof(s));
  s.F = static_cast<int>(a->frames);
  s.H = static_cast<int>(a->height);
  s.W = static_cast<int>(a->width);
  s.Cin = static_cast<int>(a->in_channels);
  s.N = static_cast<int>(a->out_channels);
  s.tw = s.W >= 32 ? 32 : (s.W >= 16 ? 16 : 8);
  int th = 128 / s.tw;
  while (th > 1 && th / 2 >= s.H) th /= 2;  // do not waste rows on short frames
  s.th = th;
  s.tf = 128 / (s.th * s.tw);
  s.fb = (s.F + s.tf - 1) / s.tf;
  s.hb = (s.H + s.th - 1) / s.th;
  s.wb = (s.W + s.tw - 1) / s.tw;
  s.boxes = s.fb * s.hb * s.wb;
  s.cblocks = s.Cin / 64;
  s.kblocks = 27 * s.cblocks;
  s.pad_front = a->causal ? 2 : 1;
  s.st = st;
  s.sh = sh;
  s.sw = sw;
  s.drop = st > 1 ? 1 : 0;
  s.Co = static_cast<int>(co);
  s.Fo = s.F * st - s.drop;
  s.Ho = s.H * sh;
  s.Wo = s.W * sw;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  // CTA pairs (two boxes per tile, M = 256) once they fill a wave of the GPU's SM pairs
  const int64_t pair_tiles = ((s.boxes + 1) / 2) * ((s.N + 255) / 256);
  const int64_t narrow_pair_tiles = ((s.boxes + 1) / 2) * ((s.N + 127) / 128);
  if (a->out_channels <= 128) {
    if (KINO_CONV_CTA_PAIRS && gemm_pairs_enabled() && narrow_pair_tiles >= device_sms() / 2) {
      if (KINO_CONV_HALO && s.W >= 128) {
        // boxes of one 128-voxel row: each input row (with its halo) serves the three kw taps
        kino::ConvShape r = s;
        r.tw = 128;
        r.th = 1;
        r.tf = 1;
        r.fb = r.F;
        r.hb = r.H;
        r.wb = (r.W + 127) / 128;
        r.boxes = r.fb * r.hb * r.wb;
        return launch_conv_2sm<128, 2, 2, 1>(a, r, strm, 23);
      }
      if (KINO_CONV_HALO && s.tf == 1 && s.th > 1)
        return launch_conv_2sm<128, 2, 2, 2>(a, s, strm, 25);
      return launch_conv_2sm<128, KINO_CONV_NARROW_STAGES, KINO_CONV_NARROW_KSUB>(a, s, strm, 8);
    }
    // narrow outputs: two boxes per tile share the weight block when that still fills the GPU
    if (KINO_CONV_PAIR_BOXES && s.boxes >= 2 * device_sms())
      return launch_conv<128, 4, 2>(a, s, strm, 7);
    return launch_conv<128, 6, 1>(a, s, strm, 4);
  }
  if (KINO_CONV_CTA_PAIRS && gemm_pairs_enabled() && pair_tiles >= device_sms() / 2) {
    if (KINO_CONV_HALO && s.W >= 128) {
      kino::ConvShape r = s;  // as for 128 channels: one 128-voxel row per box
      r.tw = 128;
      r.th = 1;
      r.tf = 1;
      r.fb = r.F;
      r.hb = r.H;
      r.wb = (r.W + 127) / 128;
      r.boxes = r.fb * r.hb * r.wb;
      return launch_conv_2sm<256, 3, 1, 1>(a, r, strm, 24);
    }
    if (KINO_CONV_HALO && s.tf == 1 && s.th > 1)
      return launch_conv_2sm<256, 3, 1, 2>(a, s, strm, 26);
    return launch_conv_2sm<256, KINO_CONV_WIDE_STAGES, KINO_CONV_WIDE_KSUB>(a, s, strm, 9);
  }
  return launch_conv<256, 4, 1>(a, s, strm, 5);
}

kino_status kino_pixel_norm(const void* x, void* out, int64_t voxels, int64_t channels, float eps,
                            int apply_silu, void* stream) {
  if (x == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_pixel_norm: null");
  if (channels % 8 || channels > 1024 || !aligned16(x) || !aligned16(out) || voxels < 1)
    return fail(KINO_ENOTSUPPORTED, "kino_pixel_norm: channels %% 8, <= 1024, aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto vec_form = [&](auto kernel, int64_t voxels_per_warp) {
    const int64_t warps = (voxels + voxels_per_warp - 1) / voxels_per_warp;
    launch_pdl(kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, st,
               static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), voxels,
               eps, apply_silu);
    return check_launch("kino_pixel_norm");
  };
  switch (channels) {
    case 64: return vec_form(kino::pixel_norm_silu_vec_kernel<64>, 4);
    case 128: return vec_form(kino::pixel_norm_silu_vec_kernel<128>, 2);
    case 256: return vec_form(kino::pixel_norm_silu_vec_kernel<256>, 1);
    case 512: return vec_form(kino::pixel_norm_silu_vec_kernel<512>, 1);
    case 1024: return vec_form(kino::pixel_norm_silu_vec_kernel<1024>, 1);
    default: break;
  }
  const int64_t threads = voxels * 32;
  const int64_t blocks = (threads + 255) / 256;
  launch_pdl(kino::pixel_norm_silu_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), voxels,
      static_cast<int>(channels), eps, apply_silu);
  return check_launch("kino_pixel_norm");
}

int64_t kino_group_norm_workspace_size(int64_t voxels, int64_t channels) {
  (void)channels;
  return (static_cast<int64_t>(gn_parts(voxels)) + 2) * kino::GN_GROUPS * sizeof(float);
}

kino_status kino_group_norm(const void* x, const void* weight, const void* bias, void* out,
                            int64_t voxels, int64_t channels, float eps, int apply_silu,
                            void* workspace, int64_t workspace_bytes, void* stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_group_norm: null operand");
  if (workspace == nullptr || workspace_bytes < kino_group_norm_workspace_size(voxels, channels))
    return fail(KINO_EINVAL, "kino_group_norm: workspace smaller than kino_group_norm_workspace_size");
  if (channels % (8 * kino::GN_GROUPS) && (channels % kino::GN_GROUPS || channels % 8))
    return fail(KINO_ENOTSUPPORTED, "kino_group_norm: channels must split into 32 groups");
  if (channels > 2048 || channels < 32 || !aligned16(x) || !aligned16(out) ||
      !aligned16(weight) || !aligned16(bias) || voxels < 1)
    return fail(KINO_ENOTSUPPORTED, "kino_group_norm: 32 <= channels <= 2048, aligned operands");
  const int parts = gn_parts(voxels);
  float* ws = static_cast<float*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const int c = static_cast<int>(channels);
  const int64_t count = voxels * (channels / kino::GN_GROUPS);
  for (int pass = 0; pass < 2; ++pass) {
    launch_pdl(kino::group_norm_partial_kernel, dim3(parts), dim3(kino::GN_THREADS), 0, s, xb, voxels, c, ws, parts,
                                                                       pass);
    launch_pdl(kino::group_norm_finalize_kernel, dim3(1), dim3(32), 0, s, ws, parts, count, eps, pass);
  }
  const int64_t blocks = gn_apply_blocks(voxels, channels);
  launch_pdl(kino::group_norm_apply_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
      xb, static_cast<const __nv_bfloat16*>(weight), static_cast<const __nv_bfloat16*>(bias),
      static_cast<__nv_bfloat16*>(out), voxels, c, ws + static_cast<int64_t>(parts) * kino::GN_GROUPS,
      ws + static_cast<int64_t>(parts) * kino::GN_GROUPS + kino::GN_GROUPS, apply_silu);
  return check_launch("kino_group_norm");
}

int64_t kino_conv3d_workspace_size(void) { return KINO_CONV_SPLIT_WORKSPACE_BYTES; }

int64_t kino_conv3d_stats_size(void) {
  // one record per TMEM lane quarter of every CTA
  return (kino::GN_STATS_RECORDS + 4 * static_cast<int64_t>(device_sms()) * 96) * 4;
}

kino_status kino_group_norm_from_stats(const void* x, const void* weight, const void* bias,
                                       void* out, int64_t voxels, int64_t channels, float eps,
                                       int apply_silu, void* stats, void* stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || out == nullptr || stats == nullptr)
    return fail(KINO_EINVAL, "kino_group_norm_from_stats: null operand");
  if (channels % kino::GN_GROUPS || channels % 8 || channels > 2048 || channels < 32 ||
      !aligned16(x) || !aligned16(out) || !aligned16(weight) || !aligned16(bias) ||
      !aligned16(stats) || voxels < 1)
    return fail(KINO_ENOTSUPPORTED,
                "kino_group_norm_from_stats: 32 <= channels <= 2048 in 32 groups, aligned operands");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* st = static_cast<float*>(stats);
  launch_pdl(kino::group_norm_merge_kernel, dim3(kino::GN_GROUPS), dim3(kino::GN_MERGE_THREADS), 0, s, st, eps);
  const int64_t blocks = gn_apply_blocks(voxels, channels);
  launch_pdl(kino::group_norm_apply_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
             static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
             static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), voxels,
             static_cast<int>(channels), static_cast<const float*>(st + 4),
             static_cast<const float*>(st + 36), apply_silu);
  return check_launch("kino_group_norm_from_stats");
}

kino_status kino_group_norm_noalloc(const void* x, const void* weight, const void* bias,
                                    void* out, int64_t voxels, int64_t channels, float eps,
                                    int apply_silu, void* stream) {
  const int64_t need = kino_group_norm_workspace_size(voxels, channels);
  if (need > KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES)
    return fail(KINO_ENOTSUPPORTED,
                "kino_group_norm_noalloc: this shape needs %lld bytes of scratch, above the "
                "static maximum of %d bytes; use kino_group_norm with a caller workspace",
                (long long)need, KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES);
  kino_status st = KINO_OK;
  void* scratch = group_norm_scratch_address(&st);
  if (scratch == nullptr) return st;
  return kino_group_norm(x, weight, bias, out, voxels, channels, eps, apply_silu, scratch,
                         KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES, stream);
}

kino_status kino_dequantize(const void* words, const void* scales, const void* biases, void* out,
                            int64_t rows, int64_t cols, int mode, int group_size, int bits,
                            int transpose_out, void* stream) {
  if (words == nullptr || scales == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_dequantize: null operand");
  if (mode < KINO_QUANT_AFFINE || mode > KINO_QUANT_NVFP4)
    return fail(KINO_EINVAL, "kino_dequantize: unknown mode %d", mode);
  if (mode == KINO_QUANT_AFFINE && biases == nullptr)
    return fail(KINO_EINVAL, "kino_dequantize: affine mode needs biases");
  const bool ok_bits = mode == KINO_QUANT_AFFINE ? (bits == 2 || bits == 4 || bits == 8)
                                                 : bits == (mode == KINO_QUANT_MXFP8 ? 8 : 4);
  const bool ok_group = mode == KINO_QUANT_AFFINE
                            ? (group_size == 32 || group_size == 64 || group_size == 128)
                            : group_size == (mode == KINO_QUANT_NVFP4 ? 16 : 32);
  if (!ok_bits || !ok_group)
    return fail(KINO_ENOTSUPPORTED, "kino_dequantize: mode %d takes neither %d bits nor groups of %d",
                mode, bits, group_size);
  if (rows < 1 || cols < 1 || cols % 16 || cols % group_size || (transpose_out && rows % 16) ||
      rows > (1ll << 31) / kino::DQ_TILE)
    return fail(KINO_ENOTSUPPORTED, "kino_dequantize: columns must be a multiple of the group size "
                                    "and of 16 (and rows of 16 for a transposed output)");
  if (!aligned16(words) || !aligned16(out))
    return fail(KINO_EINVAL, "kino_dequantize: words and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mode == KINO_QUANT_MXFP8) {
    // whole 32-code groups, grid-stride over 148 SMs x 8 CTAs
    const int64_t groups = rows * (cols / 32);
    const int64_t want = (groups + kino::DQ8_THREADS - 1) / kino::DQ8_THREADS;
    const unsigned blocks = static_cast<unsigned>(want < 148 * 8 ? want : 148 * 8);
    if (!transpose_out)
      launch_pdl(kino::dequant_mxfp8_rows_kernel, dim3(blocks), dim3(kino::DQ8_THREADS), 0, s,
                 static_cast<const uint2*>(words), static_cast<const uint8_t*>(scales),
                 static_cast<uint4*>(out), groups * 4);
    else  // rows is a multiple of 16 here
      launch_pdl(kino::dequant_mxfp8_cols_kernel, dim3(blocks), dim3(kino::DQ8_THREADS), 0, s,
                 static_cast<const uint4*>(words), static_cast<const uint8_t*>(scales),
                 static_cast<uint32_t*>(out), rows, cols);
    return check_launch("kino_dequantize");
  }
  const dim3 grid(static_cast<unsigned>((cols + kino::DQ_TILE - 1) / kino::DQ_TILE),
                  static_cast<unsigned>((rows + kino::DQ_TILE - 1) / kino::DQ_TILE));
  const uint32_t* w = static_cast<const uint32_t*>(words);
  const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(biases);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  if (bits == 8)
    launch_pdl(kino::dequant_kernel<8>, grid, dim3(kino::DQ_THREADS), 0, s, w, scales, b, o, rows,
               cols, mode, group_size, transpose_out);
  else if (bits == 4)
    launch_pdl(kino::dequant_kernel<4>, grid, dim3(kino::DQ_THREADS), 0, s, w, scales, b, o, rows,
               cols, mode, group_size, transpose_out);
  else
    launch_pdl(kino::dequant_kernel<2>, grid, dim3(kino::DQ_THREADS), 0, s, w, scales, b, o, rows,
               cols, mode, group_size, transpose_out);
  return check_launch("kino_dequantize");
}

kino_status kino_latent_to_bfhwc(const void* latent, const float* std_of_means,
                                 const float* mean_of_means, void* out, int64_t channels,
                                 int64_t voxels, void* stream) {
  if (latent == nullptr || std_of_means == nullptr || mean_of_means == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_latent_to_bfhwc: null");
  if (channels < 1 || voxels < 1) return fail(KINO_EINVAL, "kino_latent_to_bfhwc: empty");
  int64_t blocks = (channels * voxels + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  launch_pdl(kino::latent_to_bfhwc_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(latent), std_of_means, mean_of_means,
      static_cast<__nv_bfloat16*>(out), static_cast<int>(channels), voxels);
  return check_launch("kino_latent_to_bfhwc");
}

kino_status kino_tile_blend(const void* decoded, int64_t frames, int64_t height, int64_t width,
                            int64_t channels, int64_t patch, float* canvas, float* weights,
                            int64_t out_height, int64_t out_width, int64_t y0, int64_t x0,
                            const float* mask_h, const float* mask_w, void* stream) {
  if (decoded == nullptr || canvas == nullptr || weights == nullptr || mask_h == nullptr ||
      mask_w == nullptr)
    return fail(KINO_EINVAL, "kino_tile_blend: null");
  if (y0 < 0 || x0 < 0 || y0 + height * patch > out_height || x0 + width * patch > out_width)
    return fail(KINO_EINVAL, "kino_tile_blend: tile outside the canvas");
  const int64_t nrows = channels * frames * height * patch;
  if (nrows > 0x7fffffffLL || width * patch > 0x7fffffffLL || channels * patch * patch > 0x7fffffffLL)
    return fail(KINO_ENOTSUPPORTED, "kino_tile_blend: tile too large");
  int64_t blocks = nrows;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) return KINO_OK;
  launch_pdl(kino::tile_blend_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __nv_bfloat16*>(decoded), static_cast<int>(frames),
      static_cast<int>(height), static_cast<int>(width), static_cast<int>(channels),
      static_cast<int>(patch), canvas, weights, static_cast<int>(out_height),
      static_cast<int>(out_width), static_cast<int>(y0), static_cast<int>(x0), mask_h, mask_w);
  return check_launch("kino_tile_blend");
}

kino_status kino_blend_normalize(float* canvas, const float* weights, int64_t planes, int64_t hw,
                                 void* stream) {
  if (canvas == nullptr || weights == nullptr) return fail(KINO_EINVAL, "kino_blend_normalize: null");
  int64_t blocks = (planes * hw + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  launch_pdl(kino::blend_normalize_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream), canvas, weights, planes, hw);
  return check_launch("kino_blend_normalize");
}

// ---------------------------------------------------------------- peer memory
kino_status kino_peer_alloc(int64_t bytes, void** ptr, kino_ipc_handle* handle) {
  if (ptr == nullptr || handle == nullptr || bytes < 1)
    return fail(KINO_EINVAL, "kino_peer_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return fail(KINO_ECUDA, "kino_peer_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(KINO_ECUDA, "kino_peer_alloc: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
  std::memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return KINO_OK;
}

kino_status kino_peer_free(void* ptr) {
  if (ptr == nullptr) return fail(KINO_EINVAL, "kino_peer_free: null");
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(KINO_ECUDA, "kino_peer_free: %s", cudaGetErrorString(e));
  return KINO_OK;
}

kino_status kino_peer_open(const kino_ipc_handle* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(KINO_EINVAL, "kino_peer_open: null");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(KINO_ECUDA, "kino_peer_open: %s", cudaGetErrorString(e));
  return KINO_OK;
}

kino_status kino_peer_close(void* ptr) {
  if (ptr == nullptr) return fail(KINO_EINVAL, "kino_peer_close: null");
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(KINO_ECUDA, "kino_peer_close: %s", cudaGetErrorString(e));
  return KINO_OK;
}

kino_status kino_peer_barrier(void* const* flags, int64_t rank, int64_t world, int64_t epoch,
                              void* stream) {
  if (flags == nullptr) return fail(KINO_EINVAL, "kino_peer_barrier: null flags");
  if (world < 1 || world > kino::PEER_MAX_WORLD || rank < 0 || rank >= world || epoch < 1)
    return fail(KINO_EINVAL, "kino_peer_barrier: rank/world/epoch");
  launch_pdl(kino::peer_barrier_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
             reinterpret_cast<uint32_t* const*>(flags), static_cast<int>(rank),
             static_cast<int>(world), static_cast<uint32_t>(epoch));
  return check_launch("kino_peer_barrier");
}


// ---------------------------------------------------------------- fp32 parity mode
kino_status kino_linear_f32(const float* x, const float* w, float* out, int64_t batch, int64_t m,
                            int64_t n, int64_t k, int64_t ldx, int64_t bsx, int64_t ldw,
                            int64_t ldo, int64_t bso, const kino_epilogue_f32* epi,
                            void* stream) {
  if (x == nullptr || w == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_linear_f32: null operand");
  if (batch < 1 || m < 1 || n < 1 || k < 1) return fail(KINO_EINVAL, "kino_linear_f32: empty shape");
  if (k % 4 || ldx % 4 || ldw % 4 || bsx % 4 || !aligned16(x) || !aligned16(w))
    return fail(KINO_ENOTSUPPORTED, "kino_linear_f32: k and the operand strides must be multiples "
                "of 4 with 16-byte aligned operands");
  if (ldx < k || ldw < k || ldo < n) return fail(KINO_EINVAL, "kino_linear_f32: stride below width");
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL || batch > 65535 ||
      (m + kino::F32_BM - 1) / kino::F32_BM > 65535)
    return fail(KINO_ENOTSUPPORTED, "kino_linear_f32: shape too large");
  kino::F32Epi e;
  std::memset(&e, 0, sizeof(e));
  if (epi != nullptr) {
    if (epi->kind < KINO_EPI_NONE || epi->kind > KINO_EPI_EULER_X0)
      return fail(KINO_ENOTSUPPORTED, "kino_linear_f32: epilogue %d (NONE, GELU, GATED_RESIDUAL, "
                  "EULER, SIGMOID2 or EULER_X0)", epi->kind);
    if (epi->kind == KINO_EPI_GATED_RESIDUAL && (epi->residual == nullptr || epi->gate == nullptr))
      return fail(KINO_EINVAL, "kino_linear_f32: gated residual needs residual and gate");
    if ((epi->kind == KINO_EPI_EULER || epi->kind == KINO_EPI_EULER_X0) && epi->aux == nullptr)
      return fail(KINO_EINVAL, "kino_linear_f32: Euler epilogue needs the sample");
    e.kind = epi->kind;
    e.bias = epi->bias;
    e.residual = epi->residual;
    e.ld_res = epi->ld_residual;
    e.bs_res = epi->bs_residual;
    e.gate = epi->gate;
    e.bs_gate = epi->bs_gate;
    e.act_col_begin = epi->act_col_begin;
    e.scalar = epi->scalar;
    e.aux = epi->aux;
    e.ld_aux = epi->ld_aux;
    e.bs_aux = epi->bs_aux;
    e.scalar2 = epi->scalar2;
  }
  const dim3 grid(static_cast<unsigned>((n + kino::F32_BN - 1) / kino::F32_BN),
                  static_cast<unsigned>((m + kino::F32_BM - 1) / kino::F32_BM),
                  static_cast<unsigned>(batch));
  launch_pdl(kino::gemm_f32_kernel, grid, dim3(kino::F32_THREADS), 0,
             static_cast<cudaStream_t>(stream), x, w, out, static_cast<int>(m),
             static_cast<int>(n), static_cast<int>(k), ldx, bsx, ldw, ldo, bso, e);
  return check_launch("kino_linear_f32");
}

kino_status kino_attention_f32(const float* q, const float* k, const float* v, float* out,
                               int64_t batch, int64_t heads, int64_t q_tokens, int64_t kv_tokens,
                               int64_t ld_q, int64_t bs_q, int64_t ld_k, int64_t bs_k,
                               int64_t ld_v, int64_t bs_v, int64_t ld_out, int64_t bs_out,
                               float scale, const float* gate, int64_t ld_gate, int64_t bs_gate,
                               const float* key_bias, int64_t ld_key_bias, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_attention_f32: null operand");
  if (key_bias != nullptr && batch > 1 && ld_key_bias < kv_tokens)
    return fail(KINO_EINVAL, "kino_attention_f32: key bias rows shorter than the keys");
  if (gate != nullptr && ld_gate < heads)
    return fail(KINO_EINVAL, "kino_attention_f32: gate rows shorter than heads");
  if (batch < 1 || heads < 1 || q_tokens < 1 || kv_tokens < 1)
    return fail(KINO_EINVAL, "kino_attention_f32: empty shape");
  if (batch > 65535 || heads > 65535 || q_tokens > 0x7fffffffLL || kv_tokens > 0x7fffffffLL)
    return fail(KINO_ENOTSUPPORTED, "kino_attention_f32: shape too large");
  if (ld_q % 4 || ld_k % 4 || ld_v % 4 || ld_out % 4 || bs_q % 4 || bs_k % 4 || bs_v % 4 ||
      bs_out % 4 || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(KINO_ENOTSUPPORTED, "kino_attention_f32: strides must be multiples of 4 with "
                "16-byte aligned operands");
  if (ld_q < heads * 128 || ld_k < heads * 128 || ld_v < heads * 128 || ld_out < heads * 128)
    return fail(KINO_EINVAL, "kino_attention_f32: row stride below heads * 128");
  const int smem = static_cast<int>(sizeof(kino::Fa32Smem));
  kino_status st = ensure_smem(kino::attention_f32_kernel, smem, 10);
  if (st != KINO_OK) return st;
  const dim3 grid(static_cast<unsigned>((q_tokens + kino::FA32_BQ - 1) / kino::FA32_BQ),
                  static_cast<unsigned>(heads), static_cast<unsigned>(batch));
  launch_pdl(kino::attention_f32_kernel, grid, dim3(kino::FA32_THREADS), smem,
             static_cast<cudaStream_t>(stream), q, k, v, out, static_cast<int>(q_tokens),
             static_cast<int>(kv_tokens), ld_q, bs_q, ld_k, bs_k, ld_v, bs_v, ld_out, bs_out,
             scale, gate, ld_gate, bs_gate, key_bias, ld_key_bias);
  return check_launch("kino_attention_f32");
}

kino_status kino_adaln_f32(const float* x, int64_t ldx, int64_t bsx, const float* shift,
                           const float* scale, int64_t bs_mod, float* out, int64_t ldo,
                           int64_t bso, int64_t batch, int64_t rows, int64_t dim, int norm_kind,
                           float eps, void* stream) {
  if (x == nullptr || shift == nullptr || scale == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_adaln_f32: null");
  if (dim < 1 || dim > 32 * kino::ADALN32_THREADS)
    return fail(KINO_ENOTSUPPORTED, "kino_adaln_f32: dim must be 1..8192");
  if (rows < 1 || batch < 1 || batch * rows > 0x7fffffffLL)
    return fail(KINO_EINVAL, "kino_adaln_f32: rows/batch");
  if (norm_kind < KINO_NORM_RMS || norm_kind > KINO_NORM_NONE)
    return fail(KINO_EINVAL, "kino_adaln_f32: norm kind");
  launch_pdl(kino::adaln_f32_kernel, dim3(static_cast<unsigned>(batch * rows)),
             dim3(kino::ADALN32_THREADS), 0, static_cast<cudaStream_t>(stream), x, ldx, bsx,
             shift, scale, bs_mod, out, ldo, bso, static_cast<int>(rows), static_cast<int>(dim),
             norm_kind, eps);
  return check_launch("kino_adaln_f32");
}

kino_status kino_qk_norm_rope_f32(float* x, int64_t ld, int64_t bs, int64_t batch,
                                  int64_t tokens, int64_t heads, const float* weight,
                                  int norm_kind, int rope_kind, const float* cos_table,
                                  const float* sin_table, int table_batched, int64_t table_tokens,
                                  int64_t table_offset, float eps, void* stream) {
  if (x == nullptr) return fail(KINO_EINVAL, "kino_qk_norm_rope_f32: null");
  // per-head norm with pair RoPE (Flux2), or full-row norm with split RoPE (LTX-2)
  const bool flux_form = (norm_kind == KINO_QKNORM_NONE || norm_kind == KINO_QKNORM_PER_HEAD) &&
                         (rope_kind == KINO_ROPE_NONE || rope_kind == KINO_ROPE_PAIRS);
  const bool ltx_form = (norm_kind == KINO_QKNORM_NONE || norm_kind == KINO_QKNORM_FULL_ROW) &&
                        (rope_kind == KINO_ROPE_NONE || rope_kind == KINO_ROPE_SPLIT);
  if (!flux_form && !ltx_form)
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_f32: per-head norm with pair RoPE or "
                "full-row norm with split RoPE");
  if (norm_kind != KINO_QKNORM_NONE && (weight == nullptr || !aligned16(weight)))
    return fail(KINO_EINVAL, "kino_qk_norm_rope_f32: norm needs an aligned weight");
  if (rope_kind != KINO_ROPE_NONE &&
      (cos_table == nullptr || sin_table == nullptr || !aligned16(cos_table) ||
       !aligned16(sin_table)))
    return fail(KINO_EINVAL, "kino_qk_norm_rope_f32: rope needs aligned tables");
  if (ld % 4 || bs % 4 || !aligned16(x) || ld < heads * 128)
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_f32: aligned rows of heads * 128");
  if (tokens < 1 || batch < 1 || heads < 1) return fail(KINO_EINVAL, "kino_qk_norm_rope_f32: empty");
  if (rope_kind != KINO_ROPE_NONE && (table_offset < 0 || table_offset + tokens > table_tokens))
    return fail(KINO_EINVAL, "kino_qk_norm_rope_f32: table too short");
  if (tokens > 0x7fffffffLL || batch * tokens > 0x7fffffffLL)
    return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_f32: shape too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!flux_form) {
    if (heads * 64 > 256 * kino::QKROW32_MAX_PAIRS)
      return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_f32: full-row form takes rows up to 8192");
    launch_pdl(kino::qk_norm_rope_row_f32_kernel, dim3(static_cast<unsigned>(batch * tokens)),
               dim3(256), 0, st, x, ld, bs, static_cast<int>(tokens), static_cast<int>(heads),
               weight, norm_kind == KINO_QKNORM_FULL_ROW ? 1 : 0,
               rope_kind == KINO_ROPE_SPLIT ? 1 : 0, cos_table, sin_table, table_batched,
               table_tokens, table_offset, eps);
    return check_launch("kino_qk_norm_rope_f32");
  }
  const int64_t items = batch * tokens * heads;
  const int64_t blocks = (items + 7) / 8;
  if (blocks > 0x7fffffffLL) return fail(KINO_ENOTSUPPORTED, "kino_qk_norm_rope_f32: shape too large");
  launch_pdl(kino::qk_norm_rope_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
             x, ld, bs, static_cast<int>(tokens), static_cast<int>(heads), weight,
             norm_kind == KINO_QKNORM_PER_HEAD ? 1 : 0, rope_kind == KINO_ROPE_PAIRS ? 1 : 0,
             cos_table, sin_table, table_batched, table_tokens, table_offset, eps, items);
  return check_launch("kino_qk_norm_rope_f32");
}

kino_status kino_add_rows_f32(const float* a, const float* b, float* out, int64_t rows, int64_t n,
                              void* stream) {
  if (a == nullptr || b == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_add_rows_f32: null");
  if (rows < 1 || n < 1 || n > 0x7fffffffLL) return fail(KINO_EINVAL, "kino_add_rows_f32: shape");
  const int64_t total = rows * n;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::add_rows_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), a, b, out, total, static_cast<int>(n));
  return check_launch("kino_add_rows_f32");
}

static kino_status launch_elem_f32(int kind, const float* a, const float* b, float* out,
                                   int64_t n, float s0, void* stream, const char* name) {
  if (a == nullptr || out == nullptr) return fail(KINO_EINVAL, "%s: null", name);
  if (n < 0) return fail(KINO_EINVAL, "%s: negative size", name);
  if (n == 0) return KINO_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::elementwise_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), kind, a, b, out, n, s0);
  return check_launch(name);
}

kino_status kino_gelu_tanh_f32(const float* x, float* out, int64_t n, void* stream) {
  return launch_elem_f32(kino::ELEM32_GELU, x, nullptr, out, n, 0.f, stream, "kino_gelu_tanh_f32");
}

kino_status kino_silu_f32(const float* x, float* out, int64_t n, void* stream) {
  return launch_elem_f32(kino::ELEM32_SILU, x, nullptr, out, n, 0.f, stream, "kino_silu_f32");
}

kino_status kino_cfg_combine_f32(const float* cond, const float* uncond, float guidance,
                                 float* out, int64_t n, void* stream) {
  if (uncond == nullptr) return fail(KINO_EINVAL, "kino_cfg_combine_f32: null");
  return launch_elem_f32(kino::ELEM32_CFG, cond, uncond, out, n, guidance, stream,
                         "kino_cfg_combine_f32");
}

kino_status kino_euler_velocity_f32(const float* x, const float* v, float dt, float* out,
                                    int64_t n, void* stream) {
  if (v == nullptr) return fail(KINO_EINVAL, "kino_euler_velocity_f32: null");
  return launch_elem_f32(kino::ELEM32_EULER_V, x, v, out, n, dt, stream, "kino_euler_velocity_f32");
}

kino_status kino_euler_step_f32(const float* sample, const float* denoised, float ratio,
                               float* out, int64_t n, void* stream) {
  if (denoised == nullptr) return fail(KINO_EINVAL, "kino_euler_step_f32: null");
  return launch_elem_f32(kino::ELEM32_EULER_D, sample, denoised, out, n, ratio, stream,
                         "kino_euler_step_f32");
}

kino_status kino_swiglu_f32(const float* x, int64_t ldx, int64_t bsx, float* out, int64_t ldo,
                            int64_t bso, int64_t batch, int64_t rows, int64_t width,
                            void* stream) {
  if (x == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_swiglu_f32: null");
  if (batch < 1 || rows < 1 || width < 1 || width > 0x7fffffffLL || ldx < 2 * width ||
      ldo < width)
    return fail(KINO_EINVAL, "kino_swiglu_f32: shape/strides");
  const int64_t total = batch * rows * width;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::swiglu_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), x, ldx, bsx, out, ldo, bso, rows,
             static_cast<int>(width), total);
  return check_launch("kino_swiglu_f32");
}

kino_status kino_timestep_embedding_f32(const float* t, float* out, int64_t batch, int64_t dim,
                                        void* stream) {
  if (t == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_timestep_embedding_f32: null");
  if (batch < 1 || batch > 65535 || dim < 2 || dim % 2)
    return fail(KINO_EINVAL, "kino_timestep_embedding_f32: batch 1..65535, even dim");
  launch_pdl(kino::timestep_embedding_f32_kernel, dim3(static_cast<unsigned>(batch)), dim3(128),
             0, static_cast<cudaStream_t>(stream), t, out, static_cast<int>(dim));
  return check_launch("kino_timestep_embedding_f32");
}

// ---------------------------------------------------------------- video VAE, fp32 parity mode
kino_status kino_conv3d_f32(const float* x, int64_t frames, int64_t height, int64_t width,
                            int64_t in_channels, const float* weight, int64_t out_channels,
                            const float* bias, const float* residual, float* out, int causal,
                            int stride_t, int stride_h, int stride_w, void* stream) {
  if (x == nullptr || weight == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_conv3d_f32: null operand");
  if (frames < 1 || height < 1 || width < 1 || in_channels < 1 || out_channels < 1)
    return fail(KINO_EINVAL, "kino_conv3d_f32: empty shape");
  if (in_channels % 16 || !aligned16(x) || !aligned16(weight))
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d_f32: in_channels %% 16 == 0, aligned operands");
  if (stride_t < 1 || stride_t > 2 || stride_h < 1 || stride_h > 2 || stride_w < 1 || stride_w > 2)
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d_f32: depth-to-space strides of 1 or 2");
  const int64_t sub = static_cast<int64_t>(stride_t) * stride_h * stride_w;
  if (out_channels % sub) return fail(KINO_EINVAL, "kino_conv3d_f32: channels do not split into the stride");
  if (sub > 1 && residual != nullptr)
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d_f32: no residual with depth-to-space");
  const int64_t voxels = frames * height * width;
  if (voxels > 0x7fffffffLL || in_channels * 27 > 0x7fffffffLL || out_channels > 65535 * 128 ||
      (voxels + kino::F32_BM - 1) / kino::F32_BM > 65535)
    return fail(KINO_ENOTSUPPORTED, "kino_conv3d_f32: shape too large");
  kino::Conv32Shape shape;
  shape.F = static_cast<int>(frames);
  shape.H = static_cast<int>(height);
  shape.W = static_cast<int>(width);
  shape.Cin = static_cast<int>(in_channels);
  shape.N = static_cast<int>(out_channels);
  shape.causal = causal ? 1 : 0;
  shape.st = stride_t;
  shape.sh = stride_h;
  shape.sw = stride_w;
  const dim3 grid(static_cast<unsigned>((out_channels + kino::F32_BN - 1) / kino::F32_BN),
                  static_cast<unsigned>((voxels + kino::F32_BM - 1) / kino::F32_BM));
  launch_pdl(kino::conv3d_f32_kernel, grid, dim3(kino::F32_THREADS), 0,
             static_cast<cudaStream_t>(stream), x, weight, bias, residual, out, shape);
  return check_launch("kino_conv3d_f32");
}

kino_status kino_pixel_norm_f32(const float* x, float* out, int64_t voxels, int64_t channels,
                                float eps, int apply_silu, void* stream) {
  if (x == nullptr || out == nullptr) return fail(KINO_EINVAL, "kino_pixel_norm_f32: null");
  if (channels % 4 || channels < 4 || channels > 0x7fffffffLL || voxels < 1 || !aligned16(x) ||
      !aligned16(out))
    return fail(KINO_ENOTSUPPORTED, "kino_pixel_norm_f32: channels %% 4 == 0, aligned operands");
  const int64_t blocks = (voxels * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return fail(KINO_ENOTSUPPORTED, "kino_pixel_norm_f32: too many voxels");
  launch_pdl(kino::pixel_norm_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), x, out, voxels, static_cast<int>(channels), eps,
             apply_silu);
  return check_launch("kino_pixel_norm_f32");
}

kino_status kino_group_norm_f32(const float* x, const float* weight, const float* bias, float* out,
                                int64_t voxels, int64_t channels, float eps, int apply_silu,
                                void* stream) {
  if (x == nullptr || weight == nullptr || bias == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_group_norm_f32: null operand");
  if (channels % 32 || channels < 32 || channels > 0x7fffffffLL || voxels < 1)
    return fail(KINO_ENOTSUPPORTED, "kino_group_norm_f32: channels must split into 32 groups");
  launch_pdl(kino::group_norm_f32_kernel, dim3(32), dim3(kino::GN32_THREADS), 0,
             static_cast<cudaStream_t>(stream), x, weight, bias, out, voxels,
             static_cast<int>(channels), eps, apply_silu);
  return check_launch("kino_group_norm_f32");
}

kino_status kino_latent_to_bfhwc_f32(const float* latent, const float* std_of_means,
                                     const float* mean_of_means, float* out, int64_t channels,
                                     int64_t voxels, void* stream) {
  if (latent == nullptr || std_of_means == nullptr || mean_of_means == nullptr || out == nullptr)
    return fail(KINO_EINVAL, "kino_latent_to_bfhwc_f32: null");
  if (channels < 1 || channels > 0x7fffffffLL || voxels < 1)
    return fail(KINO_EINVAL, "kino_latent_to_bfhwc_f32: shape");
  int64_t blocks = (channels * voxels + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(kino::latent_to_bfhwc_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), latent, std_of_means, mean_of_means, out,
             static_cast<int>(channels), voxels);
  return check_launch("kino_latent_to_bfhwc_f32");
}

kino_status kino_tile_blend_f32(const float* decoded, int64_t frames, int64_t height, int64_t width,
                                int64_t channels, int64_t patch, float* canvas, float* weights,
                                int64_t out_height, int64_t out_width, int64_t y0, int64_t x0,
                                const float* mask_h, const float* mask_w, void* stream) {
  if (decoded == nullptr || canvas == nullptr || weights == nullptr || mask_h == nullptr ||
      mask_w == nullptr)
    return fail(KINO_EINVAL, "kino_tile_blend_f32: null");
  if (y0 < 0 || x0 < 0 || y0 + height * patch > out_height || x0 + width * patch > out_width)
    return fail(KINO_EINVAL, "kino_tile_blend_f32: tile outside the canvas");
  const int64_t nrows = channels * frames * height * patch;
  if (nrows > 0x7fffffffLL || width * patch > 0x7fffffffLL || channels * patch * patch > 0x7fffffffLL)
    return fail(KINO_ENOTSUPPORTED, "kino_tile_blend_f32: tile too large");
  int64_t blocks = nrows;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) return KINO_OK;
  launch_pdl(kino::tile_blend_kernel<float>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), decoded, static_cast<int>(frames),
             static_cast<int>(height), static_cast<int>(width), static_cast<int>(channels),
             static_cast<int>(patch), canvas, weights, static_cast<int>(out_height),
             static_cast<int>(out_width), static_cast<int>(y0), static_cast<int>(x0), mask_h,
             mask_w);
  return check_launch("kino_tile_blend_f32");
}

}  // extern "C"

#include "kino_blocks.cuh"
