// C ABI of techjam-b200: model object, packed weights, workspace carving,
// tensor-map encoding and the forward-pass launch sequence.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "tj.h"
#include "tj_attention.cuh"
#include "tj_common.cuh"
#include "tj_gemm.cuh"
#include "tj_misc.cuh"
#include "tj_poly.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

#define TJ_CUDA(call)                                                                       \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(TJ_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

#define TJ_CHECK(status) \
  do {                   \
    int s_ = (status);   \
    if (s_ != TJ_OK) return s_; \
  } while (0)

// ------------------------------------------------------------------ device info
struct DeviceInfo {
  int sms = 0;
  int major = 0;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo* out) {
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  if (g_dev[dev].sms == 0) {
    cudaDeviceProp prop;
    TJ_CUDA(cudaGetDeviceProperties(&prop, dev));
    g_dev[dev].sms = prop.multiProcessorCount;
    g_dev[dev].major = prop.major;
  }
  if (g_dev[dev].major != 10) return fail(TJ_ERR_NO_DEVICE, "device %d is sm_%d x, need sm_100", dev, g_dev[dev].major);
  *out = g_dev[dev];
  return TJ_OK;
}

// ------------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
  static std::once_flag once;
  static int status = TJ_OK;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
      status = fail(TJ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
      return;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? TJ_OK : status;
}

// fp16 row-major [rows, cols] matrix, box [box_rows, box_cols], given swizzle.
int make_map_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                 uint32_t box_cols, int swizzle_bytes) {
  TJ_CHECK(get_encoder());
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(TJ_ERR_INVALID, "tensor base not 16-byte aligned");
  if ((cols * 2) % 16 != 0) return fail(TJ_ERR_UNSUPPORTED, "row pitch %llu bytes not a multiple of 16", (unsigned long long)(cols * 2));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TJ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TJ_OK;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// 2-SM GEMM switch (TJ_PAIR_GEMM=0 turns it off, for A/B comparisons).
const bool g_use_pair_gemm = [] {
  const char* e = std::getenv("TJ_PAIR_GEMM");
  return !(e && e[0] == '0');
}();

// Persistent attention for head_dim <= 64 (the default); TJ_ATTN_PERSIST=0
// selects the one-CTA-per-pair kernel instead (A/B comparisons).
const int g_attn_persist = [] {
  const char* e = std::getenv("TJ_ATTN_PERSIST");
  return (e && e[0] == '0') ? 0 : 1;
}();

// Programmatic dependent launch for the forward-path kernels.  Every kernel
// launched this way calls griddep_wait before it reads or writes memory that
// another kernel touches; griddep_wait tracks only the preceding kernel, so
// a kernel is launched this way only when that predecessor is one of the
// forward's own kernels (the first one, after the caller's work, and every
// launch while the profiler records events between kernels, are ordinary
// launches).  Such a kernel may launch while its predecessor drains (the
// GEMMs and the persistent attention signal once their last loads are issued)
// and run its prologue -- barriers, TMEM allocation, descriptor prefetch --
// under the predecessor's tail.  That pays where kernels are short: measured
// on B200 (CUDA graphs, back to back), C2 shapes at 2 / 4 / 8 samples run
// 2.5 / 1.5 / 0.8% faster and C3 at 32 / 64 / 128 samples 6 / 3.3 / 0.7%
// faster, while the full C3 batch (256 samples) runs 1.5% slower and the full
// C2 batch is within noise.  So tj_forward enables it for B*S*d_model <= 2^24
// (C2 from 2 GPUs on, C3 from 2 GPUs on, C1).  TJ_PDL=0 / 1 forces it off /
// on (A/B comparisons); the standalone kernel entry points never use it.
std::atomic<int> g_pdl_mode{[] {
  const char* e = std::getenv("TJ_PDL");
  if (e == nullptr || e[0] == '\0') return -1;
  return e[0] == '0' ? 0 : 1;
}()};
constexpr long long kPdlMaxElems = 1LL << 24;
thread_local bool tl_pdl = false;  // launches of this thread's current forward use PDL

inline bool pdl_for(long long rows, int d_model) {
  const int mode = g_pdl_mode.load(std::memory_order_relaxed);
  return mode >= 0 ? mode == 1 : rows * d_model <= kPdlMaxElems;
}
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(tl_pdl) { tl_pdl = on; }
  ~PdlScope() { tl_pdl = prev; }
};

inline void set_pdl_attr(cudaLaunchAttribute* a) {
  a->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a->val.programmaticStreamSerializationAllowed = 1;
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  set_pdl_attr(&attr[0]);
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = tl_pdl ? 1 : 0;
  TJ_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  return TJ_OK;
}

// ------------------------------------------------------------------ kernel launchers
template <int BN, int EPI>
int launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tw, const tj::GemmParams& p, int sms, cudaStream_t st) {
  using Cfg = tj::GemmCfg<BN>;
  auto kern = tj::gemm_tc_kernel<BN, EPI>;
  static std::mutex mu;
  static bool attr_set[64] = {};
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      TJ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
      attr_set[dev] = true;
    }
  }
  const long long m_tiles = (p.M + tj::kGemmBM - 1) / tj::kGemmBM;
  const long long n_tiles = (p.N + BN - 1) / BN;
  const long long total = m_tiles * n_tiles;
  const int grid = (int)std::min<long long>(total, sms);
  if (grid <= 0) return TJ_OK;
  return launch_pdl(kern, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, st, ta, tw, p);
}

// 2-SM GEMM (cluster of 2, tcgen05 cta_group::2): grid = 2 x co-resident pairs.
template <int EPI>
int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tw, const tj::GemmParams& p, int pair_tiles,
                     cudaStream_t st) {
  using Cfg = tj::Gemm2Cfg;
  auto kern = tj::gemm_tc2_kernel<EPI>;
  static std::mutex mu;
  static int max_pairs[64] = {};
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::unique_lock<std::mutex> lock(mu);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_pairs[dev] == 0) {
    TJ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    cfg.gridDim = dim3(2);
    int n = 0;
    TJ_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_pairs[dev] = n > 0 ? n : 1;
  }
  const int pairs = std::min(pair_tiles, max_pairs[dev]);
  lock.unlock();
  if (pairs <= 0) return TJ_OK;
  cfg.gridDim = dim3(2 * pairs);
  if (tl_pdl) {
    set_pdl_attr(&attr[1]);
    cfg.numAttrs = 2;
  }
  TJ_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tw, p));
  return TJ_OK;
}

template <int EPI>
int launch_gemm(const void* a, const void* w, const tj::GemmParams& p, int sms, cudaStream_t st) {
  CUtensorMap ta, tw;
  TJ_CHECK(make_map_f16(&ta, a, p.M, p.K, tj::kGemmBM, tj::kGemmBK, 128));
  // 2-SM tiles (256 x 256 per CTA pair) when N allows and there is at least a
  // wave of them; otherwise 1-CTA tiles.
  {
    const long long m_tiles = (p.M + 127) / 128;
    const long long pair_tiles = ((m_tiles + 1) / 2) * (p.N / 256);
    // Pairs run their epilogues in lock-step; with a very short mainloop
    // (K < 512) the GELU epilogue dominates and the 1-CTA kernel is faster.
    // (At K = 512 the pair kernel measured 1% faster on C3's FFN-in once the
    // epilogue's bias loads ran a chunk ahead.)
    const bool epilogue_bound = EPI == tj::kEpiGelu && p.K < 512;
    if (g_use_pair_gemm && p.N % 256 == 0 && pair_tiles >= sms / 2 && !epilogue_bound) {
      TJ_CHECK(make_map_f16(&tw, w, p.N, p.K, 128, tj::kGemmBK, 128));
      return launch_gemm_pair<EPI>(ta, tw, p, (int)pair_tiles, st);
    }
  }
  // Wide tiles when there are enough of them to fill the machine, else 128.
  const long long m_tiles = (p.M + 127) / 128;
  const bool wide = (p.N % 256 == 0) && (m_tiles * (p.N / 256) >= sms);
  if (wide) {
    TJ_CHECK(make_map_f16(&tw, w, p.N, p.K, 256, tj::kGemmBK, 128));
    return launch_gemm_bn<256, EPI>(ta, tw, p, sms, st);
  }
  TJ_CHECK(make_map_f16(&tw, w, p.N, p.K, 128, tj::kGemmBK, 128));
  return launch_gemm_bn<128, EPI>(ta, tw, p, sms, st);
}

int launch_gemm_epi(int epi, const void* a, const void* w, const tj::GemmParams& p, int sms, cudaStream_t st) {
  switch (epi) {
    case tj::kEpiQKV: return launch_gemm<tj::kEpiQKV>(a, w, p, sms, st);
    case tj::kEpiGelu: return launch_gemm<tj::kEpiGelu>(a, w, p, sms, st);
    case tj::kEpiResid: return launch_gemm<tj::kEpiResid>(a, w, p, sms, st);
    case tj::kEpiPlain16: return launch_gemm<tj::kEpiPlain16>(a, w, p, sms, st);
    default: return fail(TJ_ERR_INVALID, "unknown epilogue %d", epi);
  }
}

template <int HD>
int launch_attn_hd(const void* q, const void* k, const void* v, const tj::AttnParams& p, int B, cudaStream_t st) {
  using Cfg = tj::AttnCfg<HD>;
  CUtensorMap tq, tk, tv;
  const uint64_t rows = (uint64_t)B * p.H * p.S;
  // K/V may hold several sequence shards of kv_shard rows (gathered by NCCL)
  const uint64_t kv_rows = (uint64_t)B * p.H * (uint64_t)p.kv_shard * (uint64_t)p.kv_shards;
  TJ_CHECK(make_map_f16(&tq, q, rows, HD, 128, Cfg::kAtomCols, Cfg::kSw));
  TJ_CHECK(make_map_f16(&tk, k, kv_rows, HD, 128, Cfg::kAtomCols, Cfg::kSw));
  TJ_CHECK(make_map_f16(&tv, v, kv_rows, HD, 128, Cfg::kAtomCols, Cfg::kSw));
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  const int q_tiles = (p.S + 127) / 128;
  const int n_pairs = (q_tiles + 1) / 2;
  bool persistent = false;
  if constexpr (Cfg::kPSeparate) persistent = g_attn_persist != 0;
  if (persistent) {
    if constexpr (Cfg::kPSeparate) {
      // one CTA per SM over a heavy-first list of (pair, head, sample) items
      using PC = tj::AttnPCfg<HD>;
      auto kern = tj::attn_fwd_persistent_kernel<HD>;
      static std::mutex mu;
      static bool checked[64] = {};
      {
        std::lock_guard<std::mutex> lock(mu);
        if (!checked[dev]) {
          // The kernel's per-warpgroup register budgets (setmaxnreg) add up to
          // exactly the registers a 384-thread CTA is launched with; any other
          // launch register count would leave the softmax warps waiting for
          // registers that never free up, so refuse to launch instead.
          cudaFuncAttributes fa;
          TJ_CUDA(cudaFuncGetAttributes(&fa, kern));
          if (fa.numRegs != PC::kRegLaunch)
            return fail(TJ_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, needs %d",
                        fa.numRegs, PC::kRegLaunch);
          TJ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::kSmemBytes));
          checked[dev] = true;
        }
      }
      DeviceInfo di;
      TJ_CHECK(device_info(&di));
      const long long items = (long long)n_pairs * B * p.H;
      if (items > 0x7fffffffLL - 2LL * di.sms) return fail(TJ_ERR_UNSUPPORTED, "too many attention work items");
      const int grid = (int)std::min<long long>(items, di.sms);
      if (grid <= 0) return TJ_OK;
      TJ_CHECK(launch_pdl(kern, dim3(grid), dim3(PC::kThreads), PC::kSmemBytes, st, tq, tk, tv, p, n_pairs));
    }
  } else {
    static std::mutex mu;
    static bool attr_set[64] = {};
    auto kern = tj::attn_fwd_kernel<HD>;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (!attr_set[dev]) {
        TJ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
        attr_set[dev] = true;
      }
    }
    dim3 grid(n_pairs, B * p.H);  // one CTA per pair of 128-query tiles
    TJ_CHECK(launch_pdl(kern, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, st, tq, tk, tv, p));
  }
  TJ_CUDA(cudaGetLastError());
  return TJ_OK;
}

int launch_attention(const void* q, const void* k, const void* v, int head_dim, const tj::AttnParams& p, int B,
                     cudaStream_t st) {
  if (B <= 0 || p.S <= 0) return TJ_OK;
  if ((long long)B * p.H > 65535) return fail(TJ_ERR_UNSUPPORTED, "batch*heads %lld exceeds 65535", (long long)B * p.H);
  switch (head_dim) {
    case 32: return launch_attn_hd<32>(q, k, v, p, B, st);
    case 64: return launch_attn_hd<64>(q, k, v, p, B, st);
    case 128: return launch_attn_hd<128>(q, k, v, p, B, st);
    default: return fail(TJ_ERR_UNSUPPORTED, "head_dim %d not supported (32, 64, 128)", head_dim);
  }
}

int launch_layernorm(const float* x, const float* g, const float* b, void* out, bool f16, bool all_rows, int d,
                     float eps, const tj::RowValidity& rv, const uint8_t* tile_live, cudaStream_t st) {
  if (d % 4 != 0 || d > 4096) return fail(TJ_ERR_UNSUPPORTED, "LayerNorm width %d (need multiple of 4, <= 4096)", d);
  if (rv.M == 0) return TJ_OK;
  const int warps = 4;
  const long long blocks = (rv.M + warps - 1) / warps;
  if (blocks > 0x7fffffffLL) return fail(TJ_ERR_UNSUPPORTED, "too many rows");
  const int vpl = (d / 4 + 31) / 32;
#define TJ_LN(V)                                                                                              \
  if (f16) {                                                                                                  \
    if (all_rows) TJ_CHECK(launch_pdl(tj::layernorm_kernel<V, true, true>, dim3((unsigned)blocks), dim3(32 * warps), 0, st, x, g, b, out, d, eps, rv, tile_live)); \
    else TJ_CHECK(launch_pdl(tj::layernorm_kernel<V, true, false>, dim3((unsigned)blocks), dim3(32 * warps), 0, st, x, g, b, out, d, eps, rv, tile_live));         \
  } else {                                                                                                    \
    if (all_rows) TJ_CHECK(launch_pdl(tj::layernorm_kernel<V, false, true>, dim3((unsigned)blocks), dim3(32 * warps), 0, st, x, g, b, out, d, eps, rv, tile_live)); \
    else TJ_CHECK(launch_pdl(tj::layernorm_kernel<V, false, false>, dim3((unsigned)blocks), dim3(32 * warps), 0, st, x, g, b, out, d, eps, rv, tile_live));        \
  }
  if (vpl <= 1) { TJ_LN(1) }
  else if (vpl <= 2) { TJ_LN(2) }
  else if (vpl <= 4) { TJ_LN(4) }
  else if (vpl <= 8) { TJ_LN(8) }
  else { TJ_LN(32) }
#undef TJ_LN
  TJ_CUDA(cudaGetLastError());
  return TJ_OK;
}

// Mask -> per-sample lengths / flags and the live 128-row tiles.  With
// counts/row_of/pack_of (varlen packing) the tiles are those of the packed
// valid tokens and row_of / pack_of map packed rows to padded rows and back.
int launch_prepare(const uint8_t* mask, int B, int S, int* lengths, uint8_t* general, int* tile_list, int* n_live,
                   uint8_t* tile_live, int* sched, int* counts, int* row_of, int* pack_of, cudaStream_t st) {
  {
    // The stream's previous work is the caller's (a copy, a memset, an event,
    // another library's kernel), which griddepcontrol.wait does not track:
    // the forward's first kernel is an ordinary launch that waits for all of it.
    const PdlScope first(false);
    TJ_CHECK(launch_pdl(tj::prep_lengths_kernel, dim3(B), dim3(1024), 0, st, mask, S, lengths, general, sched,
                        counts));
  }
  if (row_of != nullptr) {
    TJ_CHECK(launch_pdl(tj::prep_pack_kernel, dim3(B), dim3(1024), 0, st, mask, S, lengths, general, counts, pack_of,
                        row_of));
    const int n_tiles = (int)(((long long)B * S + 127) / 128);
    return launch_pdl(tj::prep_pack_tiles_kernel, dim3(1), dim3(1024), 0, st, counts, B, row_of, tile_list, n_live,
                      tile_live, n_tiles);
  }
  return launch_pdl(tj::prep_tiles_kernel, dim3(1), dim3(1024), 0, st, lengths, B, S, tile_list, n_live, tile_live);
}

// ------------------------------------------------------------------ workspace layout
struct Workspace {
  int* lengths;
  uint8_t* general;
  int* tile_list;
  int* n_live;
  uint8_t* tile_live;
  int* sched;   // attention work scheduler (2 ints, zeroed by the mask prep)
  int* counts;  // [B] valid tokens per sample
  int* row_of;  // [M] padded row of each packed row (varlen packing)
  int* pack_of; // [M] packed row of each padded row, -1 for padding
  __half* act;  // [M, d]: LN output, then attention context (reused)
  __half* q;
  __half* k;
  __half* v;    // [B, H, S, hd] each
  __half* ff;   // [M, F]
  tj::PolyCtl* poly_ctl;  // polynomial route (null when the route cannot run)
  __half* poly_snap;
  __half* poly_kt;        // K transposed [B, H, 64, S] for the polynomial update
};

// Exact prefix of the polynomial route (the reference's EXACT_PREFIX) and the
// shortest sequence TJ_ROUTE_AUTO sends down that route.
constexpr int kPolyExactPrefix = 4096;
constexpr int kPolyAutoMinSeq = 16384;

// Can the polynomial route run for this shape under this route request?
bool poly_eligible(const TjConfig& c, int S, int route) {
  if (route == TJ_ROUTE_EXACT || !c.causal || c.d_model / c.num_heads != 64) return false;
  if (S % tj::kPolyChunk != 0 || S <= kPolyExactPrefix) return false;
  return route == TJ_ROUTE_POLY || S >= kPolyAutoMinSeq;
}

size_t poly_snap_elems(int BH, int S) {
  const size_t n_snap = (size_t)(S / tj::kPolyChunk - kPolyExactPrefix / tj::kPolyChunk);
  return (size_t)BH * n_snap * tj::kPolyN * tj::kPolyFeat;
}

size_t carve(const TjConfig& c, int B, int S, int route, uint8_t* base, Workspace* w) {
  const size_t M = (size_t)B * S;
  const size_t tiles = (M + 127) / 128;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  Workspace t;
  t.lengths = reinterpret_cast<int*>(take(sizeof(int) * B));
  t.general = take(B);
  t.tile_list = reinterpret_cast<int*>(take(sizeof(int) * tiles));
  t.n_live = reinterpret_cast<int*>(take(sizeof(int)));
  t.tile_live = take(tiles);
  t.sched = reinterpret_cast<int*>(take(2 * sizeof(int)));
  t.counts = reinterpret_cast<int*>(take(sizeof(int) * B));
  t.row_of = reinterpret_cast<int*>(take(sizeof(int) * M));
  t.pack_of = reinterpret_cast<int*>(take(sizeof(int) * M));
  t.act = reinterpret_cast<__half*>(take(2 * M * c.d_model));
  t.q = reinterpret_cast<__half*>(take(2 * M * c.d_model));
  t.k = reinterpret_cast<__half*>(take(2 * M * c.d_model));
  t.v = reinterpret_cast<__half*>(take(2 * M * c.d_model));
  t.ff = reinterpret_cast<__half*>(take(2 * M * c.ffn_dim));
  t.poly_ctl = nullptr;
  t.poly_snap = nullptr;
  t.poly_kt = nullptr;
  if (poly_eligible(c, S, route)) {
    t.poly_ctl = reinterpret_cast<tj::PolyCtl*>(take(sizeof(tj::PolyCtl)));
    t.poly_snap = reinterpret_cast<__half*>(take(2 * poly_snap_elems(B * c.num_heads, S)));
    t.poly_kt = reinterpret_cast<__half*>(take(2 * (size_t)B * c.num_heads * 64 * S));
  }
  if (w) *w = t;
  return off;
}

}  // namespace

// ------------------------------------------------------------------ model object
struct TjLayerPacked {
  __half* wqkv;  // [3d, d]
  __half* wo;    // [d, d]
  __half* w1;    // [F, d]
  __half* w2;    // [d, F]
  float* bqkv;   // [3d]
  float* bo;
  float* b1;
  float* b2;
  float* ln1_g;
  float* ln1_b;
  float* ln2_g;
  float* ln2_b;
};

struct TjModel {
  TjConfig cfg;
  int device;
  std::vector<TjLayerPacked> layers;
  float* final_g = nullptr;
  float* final_b = nullptr;
  void* weights = nullptr;  // single allocation for all packed parameters
  int* err = nullptr;       // device error word
  long long launches = 0;   // kernels launched through this model
  // per-launch event profiling (tj_profile_begin / tj_profile_end)
  bool prof_on = false;
  int prof_max = 0;
  int prof_n = 0;
  std::vector<cudaEvent_t> prof_ev;  // 2 per launch
  std::vector<int> prof_cls;
  // Sequence-sharded polynomial route: the guard's verdict per layer, taken on
  // the first forward of a shard shape and reused after it, as the reference
  // estimates sigma once per attention module and caches it
  // (src/implementations/extreme.py:297-301).  -1: not yet evaluated.
  tj::PolyCtl* shard_ctl = nullptr;   // [num_layers] device copies of the guard result
  std::vector<int> shard_route;        // host copy of each layer's admit flag
  long long shard_key[3] = {0, 0, 0};  // batch, seq_local, world of the cached verdicts
};

namespace {
// Event record that also works while the stream is being captured into a CUDA
// graph: there it becomes an event-record node, re-recorded at every replay.
int record_event(cudaEvent_t ev, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  TJ_CUDA(cudaStreamIsCapturing(st, &cs));
  TJ_CUDA(cudaEventRecordWithFlags(ev, st, cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal
                                                                              : cudaEventRecordDefault));
  return TJ_OK;
}
// Runs one launcher, counting its kernels and bracketing it with an event pair
// when profiling is active.
template <class F>
int timed_launch(TjModel* m, int cls, int kernels, cudaStream_t st, F&& launch) {
  if (m == nullptr) return launch();  // building-block call: no model to count or profile
  const bool rec = m->prof_on && m->prof_n < m->prof_max;
  if (rec) TJ_CHECK(record_event(m->prof_ev[2 * m->prof_n], st));
  const int s = launch();
  if (s != TJ_OK) return s;
  m->launches += kernels;
  if (rec) {
    TJ_CHECK(record_event(m->prof_ev[2 * m->prof_n + 1], st));
    m->prof_cls[m->prof_n] = cls;
    ++m->prof_n;
  }
  return TJ_OK;
}
// Polynomial route for one layer: guard -> (exact prefix | whole sequence if
// not admitted) on the flash kernel -> state update -> apply.  All admission
// decisions stay on the device.
// K^T and the update kernel (shared by the single-GPU and the sequence-sharded routes).
int launch_poly_update(const tj::PolyParams& pp, const CUtensorMap& tv, cudaStream_t st) {
  const int BH = pp.B * pp.H;
  tj::poly_k_transpose_kernel<<<dim3(pp.S / 64, BH), 256, 0, st>>>(pp.k, pp.kt, pp.S);
  TJ_CUDA(cudaGetLastError());
  CUtensorMap tkt;
  TJ_CHECK(make_map_f16(&tkt, pp.kt, (uint64_t)BH * 64, (uint64_t)pp.S, 64, 64, 128));
  tj::poly_update_kernel<<<dim3(tj::kPolyFeatBlocks, BH), 192, tj::kUpdSmem, st>>>(tkt, tv, pp);
  TJ_CUDA(cudaGetLastError());
  return TJ_OK;
}

int launch_poly_route(const __half* q, const __half* k, const __half* v, __half* ctx, const int* lengths, int B,
                      int H, int S, int d_model, int exact_prefix, tj::PolyCtl* ctl, __half* snap, __half* kt,
                      TjModel* m, const tj::AttnParams& ap_in, cudaStream_t st) {
  tj::PolyParams pp{};
  pp.q = q; pp.k = k; pp.v = v; pp.ctx = ctx; pp.snap = snap; pp.kt = kt; pp.ctl = ctl; pp.lengths = lengths;
  pp.B = B; pp.H = H; pp.S = S; pp.d_model = d_model;
  pp.prefix_chunks = exact_prefix / tj::kPolyChunk;
  pp.scale = 0.125f;  // 64^-0.5
  pp.err = ap_in.err;
  pp.S_total = S;
  pp.t_before = 0.f;
  pp.total = nullptr;
  pp.all_chunks = 0;
  pp.guard_shards = 1;
  const int n_chunks = S / tj::kPolyChunk;
  if (pp.prefix_chunks < 1 || pp.prefix_chunks >= n_chunks || exact_prefix % tj::kPolyChunk)
    return fail(TJ_ERR_UNSUPPORTED, "polynomial route needs 512 <= exact prefix < seq_len, multiple of 512");
  TJ_CHECK(timed_launch(m, TJ_K_POLY, 2, st, [&]() -> int {
    TJ_CUDA(cudaMemsetAsync(ctl, 0, sizeof(tj::PolyCtl), st));
    tj::poly_guard_kernel<<<dim3(tj::kPolySample / 64, B * H), 256, 0, st>>>(pp);
    TJ_CUDA(cudaGetLastError());
    tj::poly_guard_finalize<<<1, 1, 0, st>>>(pp);
    TJ_CUDA(cudaGetLastError());
    return TJ_OK;
  }));
  tj::AttnParams ap = ap_in;
  ap.poly_admit = &ctl->admit;
  ap.exact_pairs = exact_prefix / 256;
  if (ap.sched == nullptr) ap.sched = ctl->sched;
  TJ_CHECK(timed_launch(m, TJ_K_ATTN, 1, st, [&] { return launch_attention(q, k, v, 64, ap, B, st); }));
  const uint64_t rows = (uint64_t)B * H * S;
  CUtensorMap tq, tk, tv, tsn;
  TJ_CHECK(make_map_f16(&tq, q, rows, 64, 128, 64, 128));
  TJ_CHECK(make_map_f16(&tk, k, rows, 64, 128, 64, 128));
  TJ_CHECK(make_map_f16(&tv, v, rows, 64, 128, 64, 128));
  const uint64_t snap_rows = (uint64_t)B * H * (n_chunks - pp.prefix_chunks) * tj::kPolyN;
  TJ_CHECK(make_map_f16(&tsn, snap, snap_rows, tj::kPolyFeat, tj::kPolyN, 64, 128));
  static std::mutex mu;
  static bool attr_set[64] = {};
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      TJ_CUDA(cudaFuncSetAttribute(tj::poly_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tj::kUpdSmem));
      TJ_CUDA(cudaFuncSetAttribute(tj::poly_apply_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tj::kAppSmem));
      attr_set[dev] = true;
    }
  }
  TJ_CHECK(timed_launch(m, TJ_K_POLY, 2, st, [&]() -> int { return launch_poly_update(pp, tv, st); }));
  TJ_CHECK(timed_launch(m, TJ_K_POLY, 1, st, [&]() -> int {
    tj::poly_apply_kernel<<<dim3((n_chunks - pp.prefix_chunks) * 4, B * H), tj::kAppThreads, tj::kAppSmem, st>>>(tq, tk, tv, tsn,
                                                                                                   pp);
    TJ_CUDA(cudaGetLastError());
    return TJ_OK;
  }));
  return TJ_OK;
}

}  // namespace

extern "C" {

int tj_version(void) { return 1; }

const char* tj_last_error(void) { return g_last_error.c_str(); }

int tj_model_create(const TjConfig* cfg, TjModel** out) {
  if (!cfg || !out) return fail(TJ_ERR_INVALID, "null argument");
  *out = nullptr;
  const TjConfig c = *cfg;
  if (c.d_model <= 0 || c.num_heads <= 0 || c.ffn_dim <= 0 || c.num_layers <= 0)
    return fail(TJ_ERR_INVALID, "config fields must be positive");
  if (c.d_model % c.num_heads) return fail(TJ_ERR_INVALID, "d_model %% num_heads != 0");
  const int hd = c.d_model / c.num_heads;
  if (hd != 32 && hd != 64 && hd != 128) return fail(TJ_ERR_UNSUPPORTED, "head_dim %d not supported (32, 64, 128)", hd);
  if (c.d_model % 64 || c.ffn_dim % 64) return fail(TJ_ERR_UNSUPPORTED, "d_model and ffn_dim must be multiples of 64");
  if (c.d_model > 4096) return fail(TJ_ERR_UNSUPPORTED, "d_model > 4096");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  TjModel* m = new TjModel();
  m->cfg = c;
  if (m->cfg.layer_norm_eps <= 0.f) m->cfg.layer_norm_eps = 1e-5f;
  TJ_CUDA(cudaGetDevice(&m->device));
  const size_t d = c.d_model, F = c.ffn_dim;
  const size_t per_layer = align_up(2 * 3 * d * d, 256) + align_up(2 * d * d, 256) + align_up(2 * F * d, 256) +
                           align_up(2 * d * F, 256) + align_up(4 * 3 * d, 256) + 3 * align_up(4 * d, 256) +
                           align_up(4 * F, 256) + 4 * align_up(4 * d, 256);
  const size_t total = per_layer * c.num_layers + 2 * align_up(4 * d, 256) + 256;
  cudaError_t e = cudaMalloc(&m->weights, total);
  if (e != cudaSuccess) { delete m; return fail(TJ_ERR_CUDA, "cudaMalloc weights: %s", cudaGetErrorString(e)); }
  e = cudaMalloc(&m->err, sizeof(int));
  if (e != cudaSuccess) { cudaFree(m->weights); delete m; return fail(TJ_ERR_CUDA, "cudaMalloc err: %s", cudaGetErrorString(e)); }
  cudaMemset(m->err, 0, sizeof(int));
  e = cudaMalloc(&m->shard_ctl, sizeof(tj::PolyCtl) * c.num_layers);
  if (e != cudaSuccess) {
    cudaFree(m->weights); cudaFree(m->err); delete m;
    return fail(TJ_ERR_CUDA, "cudaMalloc guard cache: %s", cudaGetErrorString(e));
  }
  m->shard_route.assign(c.num_layers, -1);
  uint8_t* p = static_cast<uint8_t*>(m->weights);
  auto take = [&](size_t bytes) { uint8_t* r = p; p += align_up(bytes, 256); return r; };
  m->layers.resize(c.num_layers);
  for (auto& L : m->layers) {
    L.wqkv = reinterpret_cast<__half*>(take(2 * 3 * d * d));
    L.wo = reinterpret_cast<__half*>(take(2 * d * d));
    L.w1 = reinterpret_cast<__half*>(take(2 * F * d));
    L.w2 = reinterpret_cast<__half*>(take(2 * d * F));
    L.bqkv = reinterpret_cast<float*>(take(4 * 3 * d));
    L.bo = reinterpret_cast<float*>(take(4 * d));
    L.b2 = reinterpret_cast<float*>(take(4 * d));
    L.ln1_g = reinterpret_cast<float*>(take(4 * d));
    L.b1 = reinterpret_cast<float*>(take(4 * F));
    L.ln1_b = reinterpret_cast<float*>(take(4 * d));
    L.ln2_g = reinterpret_cast<float*>(take(4 * d));
    L.ln2_b = reinterpret_cast<float*>(take(4 * d));
  }
  m->final_g = reinterpret_cast<float*>(take(4 * d));
  m->final_b = reinterpret_cast<float*>(take(4 * d));
  *out = m;
  return TJ_OK;
}

int tj_model_destroy(TjModel* m) {
  if (!m) return TJ_OK;
  for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
  cudaFree(m->weights);
  cudaFree(m->err);
  cudaFree(m->shard_ctl);
  delete m;
  return TJ_OK;
}

static int convert(const float* src, __half* dst, size_t n, cudaStream_t st) {
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 4096);
  tj::f32_to_f16_kernel<<<blocks, 256, 0, st>>>(src, dst, (long long)n);
  TJ_CUDA(cudaGetLastError());
  return TJ_OK;
}

int tj_model_load_layer(TjModel* m, int layer, const TjLayerParams* P, void* stream) {
  if (!m || !P) return fail(TJ_ERR_INVALID, "null argument");
  if (layer < 0 || layer >= m->cfg.num_layers) return fail(TJ_ERR_INVALID, "layer %d out of range", layer);
  const void* ptrs[] = {P->norm1_weight, P->norm1_bias, P->q_weight, P->q_bias, P->k_weight, P->k_bias,
                        P->v_weight, P->v_bias, P->out_weight, P->out_bias, P->norm2_weight, P->norm2_bias,
                        P->ffn_in_weight, P->ffn_in_bias, P->ffn_out_weight, P->ffn_out_bias};
  for (const void* q : ptrs)
    if (!q) return fail(TJ_ERR_INVALID, "null parameter pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t d = m->cfg.d_model, F = m->cfg.ffn_dim;
  TjLayerPacked& L = m->layers[layer];
  m->shard_route[layer] = -1;  // new weights: the layer's guard verdict is re-evaluated
  TJ_CHECK(convert(P->q_weight, L.wqkv, d * d, st));
  TJ_CHECK(convert(P->k_weight, L.wqkv + d * d, d * d, st));
  TJ_CHECK(convert(P->v_weight, L.wqkv + 2 * d * d, d * d, st));
  TJ_CHECK(convert(P->out_weight, L.wo, d * d, st));
  TJ_CHECK(convert(P->ffn_in_weight, L.w1, F * d, st));
  TJ_CHECK(convert(P->ffn_out_weight, L.w2, d * F, st));
  TJ_CUDA(cudaMemcpyAsync(L.bqkv, P->q_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.bqkv + d, P->k_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.bqkv + 2 * d, P->v_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.bo, P->out_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.b1, P->ffn_in_bias, 4 * F, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.b2, P->ffn_out_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.ln1_g, P->norm1_weight, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.ln1_b, P->norm1_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.ln2_g, P->norm2_weight, 4 * d, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(L.ln2_b, P->norm2_bias, 4 * d, cudaMemcpyDeviceToDevice, st));
  return TJ_OK;
}

int tj_model_load_final_norm(TjModel* m, const float* w, const float* b, void* stream) {
  if (!m || !w || !b) return fail(TJ_ERR_INVALID, "null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TJ_CUDA(cudaMemcpyAsync(m->final_g, w, 4 * (size_t)m->cfg.d_model, cudaMemcpyDeviceToDevice, st));
  TJ_CUDA(cudaMemcpyAsync(m->final_b, b, 4 * (size_t)m->cfg.d_model, cudaMemcpyDeviceToDevice, st));
  return TJ_OK;
}

int tj_workspace_bytes(const TjModel* m, int B, int S, int route, size_t* bytes) {
  if (!m || !bytes) return fail(TJ_ERR_INVALID, "null argument");
  if (B < 0 || S < 0) return fail(TJ_ERR_INVALID, "negative shape");
  *bytes = carve(m->cfg, B, S, route, nullptr, nullptr);
  return TJ_OK;
}

int tj_device_error(TjModel* m, int* code) {
  if (!m || !code) return fail(TJ_ERR_INVALID, "null argument");
  TJ_CUDA(cudaMemcpy(code, m->err, sizeof(int), cudaMemcpyDeviceToHost));
  TJ_CUDA(cudaMemset(m->err, 0, sizeof(int)));
  return TJ_OK;
}

int tj_forward(TjModel* m, const float* x, const uint8_t* mask, float* out, int B, int S, int route, void* ws,
               size_t ws_bytes, void* stream) {
  if (!m || !x || !out || !ws) return fail(TJ_ERR_INVALID, "null argument");
  if (B <= 0 || S <= 0) return fail(TJ_ERR_INVALID, "batch and seq_len must be positive");
  if (x == out) return fail(TJ_ERR_INVALID, "x and out must not alias");
  if (route != TJ_ROUTE_EXACT && route != TJ_ROUTE_AUTO && route != TJ_ROUTE_POLY)
    return fail(TJ_ERR_INVALID, "unknown attention route %d", route);
  const TjConfig& c = m->cfg;
  const size_t need = carve(c, B, S, route, nullptr, nullptr);
  if (ws_bytes < need) return fail(TJ_ERR_INVALID, "workspace %zu bytes < required %zu", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return fail(TJ_ERR_INVALID, "workspace not 256-byte aligned");
  if ((long long)B * S > (1LL << 31) / 128) return fail(TJ_ERR_UNSUPPORTED, "batch*seq_len too large");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev != m->device) return fail(TJ_ERR_INVALID, "model lives on device %d, current device is %d", m->device, dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Workspace w;
  carve(c, B, S, route, static_cast<uint8_t*>(ws), &w);
  const int d = c.d_model, H = c.num_heads, hd = d / H, F = c.ffn_dim;
  const int M = B * S;
  // the profiler's event records sit between the launches: no PDL there
  const PdlScope pdl_scope(pdl_for(M, d) && !m->prof_on);

  // Varlen token packing: with padding present (a mask) the LayerNorm
  // outputs, the GEMMs' fp16 rows and the attention context hold only the
  // valid tokens, back to back; the FP32 residual stream, Q/K/V and the output
  // keep the padded [B, S] layout (the polynomial route, for unpadded long
  // sequences only, keeps the padded rows throughout).
  const bool packed = mask != nullptr && w.poly_ctl == nullptr;
  TJ_CHECK(timed_launch(m, TJ_K_PREP, packed ? 3 : 2, st, [&] {
    return launch_prepare(mask, B, S, w.lengths, w.general, w.tile_list, w.n_live, w.tile_live, w.sched, w.counts,
                          packed ? w.row_of : nullptr, w.pack_of, st);
  }));
  tj::RowValidity rv{w.lengths, mask, S, (long long)M, packed ? w.pack_of : nullptr};
  tj::RowValidity rv_out{w.lengths, mask, S, (long long)M, nullptr};  // final LayerNorm: every padded row

  tj::GemmParams gp{};
  gp.M = M;
  gp.seq = S;
  gp.lengths = w.lengths;
  gp.mask = mask;
  gp.tile_list = w.tile_list;
  gp.n_live = w.n_live;
  gp.q = w.q; gp.k = w.k; gp.v = w.v;
  gp.heads = H; gp.head_dim = hd; gp.d_model = d;
  gp.err = m->err;
  gp.row_of = packed ? w.row_of : nullptr;

  tj::AttnParams ap{};
  ap.pack_of = packed ? w.pack_of : nullptr;
  ap.lengths = w.lengths;
  ap.mask = mask;
  ap.general = w.general;
  ap.ctx = w.act;
  ap.S = S; ap.H = H; ap.d_model = d;
  ap.causal = c.causal ? 1 : 0;
  ap.scale_log2 = (float)(1.0 / std::sqrt((double)hd) * 1.4426950408889634);
  ap.err = m->err;
  ap.q_pos0 = 0;
  ap.kv_shard = S;
  ap.kv_shards = 1;
  ap.B = B;
  ap.sched = w.sched;

  const float eps = c.layer_norm_eps;
  const float* resid_in = x;
  for (int l = 0; l < c.num_layers; ++l) {
    const TjLayerPacked& L = m->layers[l];
    // LN1 -> act (fp16)
    TJ_CHECK(timed_launch(m, TJ_K_LN, 1, st, [&] {
      return launch_layernorm(resid_in, L.ln1_g, L.ln1_b, w.act, true, false, d, eps, rv, w.tile_live, st);
    }));
    // packed QKV projection -> Q, K, V [B, H, S, hd]
    gp.N = 3 * d; gp.K = d; gp.bias = L.bqkv;
    TJ_CHECK(timed_launch(m, TJ_K_QKV, 1, st, [&] { return launch_gemm_epi(tj::kEpiQKV, w.act, L.wqkv, gp, di.sms, st); }));
    // attention -> ctx (reuses act): exact flash, or the guarded polynomial
    // route (device-side guard; the flash kernel then covers the exact prefix)
    if (w.poly_ctl != nullptr) {
      TJ_CHECK(launch_poly_route(w.q, w.k, w.v, w.act, w.lengths, B, H, S, d, kPolyExactPrefix, w.poly_ctl,
                                 w.poly_snap, w.poly_kt, m, ap, st));
    } else {
      TJ_CHECK(timed_launch(m, TJ_K_ATTN, 1, st, [&] { return launch_attention(w.q, w.k, w.v, hd, ap, B, st); }));
    }
    // out projection + residual -> out (fp32 residual stream)
    gp.N = d; gp.K = d; gp.bias = L.bo; gp.out32 = out; gp.resid = resid_in;
    TJ_CHECK(timed_launch(m, TJ_K_OUT, 1, st, [&] { return launch_gemm_epi(tj::kEpiResid, w.act, L.wo, gp, di.sms, st); }));
    // LN2 -> act
    TJ_CHECK(timed_launch(m, TJ_K_LN, 1, st, [&] {
      return launch_layernorm(out, L.ln2_g, L.ln2_b, w.act, true, false, d, eps, rv, w.tile_live, st);
    }));
    // FFN in + GELU -> ff
    gp.N = F; gp.K = d; gp.bias = L.b1; gp.out16 = w.ff;
    TJ_CHECK(timed_launch(m, TJ_K_FFN_IN, 1, st, [&] { return launch_gemm_epi(tj::kEpiGelu, w.act, L.w1, gp, di.sms, st); }));
    // FFN out + residual (in place) -> out
    gp.N = d; gp.K = F; gp.bias = L.b2; gp.out32 = out; gp.resid = out;
    TJ_CHECK(timed_launch(m, TJ_K_FFN_OUT, 1, st, [&] { return launch_gemm_epi(tj::kEpiResid, w.ff, L.w2, gp, di.sms, st); }));
    resid_in = out;
  }
  // final LayerNorm in place; every invalid row becomes exactly 0
  TJ_CHECK(timed_launch(m, TJ_K_LN_FINAL, 1, st, [&] {
    return launch_layernorm(out, m->final_g, m->final_b, out, false, true, d, eps, rv_out, w.tile_live, st);
  }));
  return TJ_OK;
}

// ------------------------------------------------------------------ allocation-free forward
// Some callers cannot call cudaMalloc on their call path: a host application
// or serving runtime that owns a fixed device-memory budget and forbids
// allocation after start-up, or a latency-critical path where cudaMalloc's
// implicit device synchronisation is not acceptable.  tj_forward_noalloc
// gives them the same forward with its scratch in this fixed array, so the
// call itself allocates nothing.  Every device that loads this library holds
// the array (TJ_NOALLOC_SCRATCH_BYTES) until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[TJ_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Host code cannot use g_noalloc_scratch's name as a device pointer (it is a
// host-side stand-in); resolve the real address once per device, with that
// device current.  The cached address belongs to the device's current
// context: after cudaDeviceReset (which destroys it) the library must be
// reloaded before tj_forward_noalloc is used on that device again.
int noalloc_scratch(void** out) {
  int dev = 0;
  TJ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(TJ_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(TJ_ERR_CUDA, "cudaGetSymbolAddress(noalloc scratch): %s", cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return TJ_OK;
}
}  // namespace

int tj_forward_noalloc(TjModel* m, const float* x, const uint8_t* mask, float* out, int B, int S, int route,
                       void* stream) {
  if (!m) return fail(TJ_ERR_INVALID, "null model");
  if (B <= 0 || S <= 0) return fail(TJ_ERR_INVALID, "batch and seq_len must be positive");
  const size_t need = carve(m->cfg, B, S, route, nullptr, nullptr);
  if (need > (size_t)TJ_NOALLOC_SCRATCH_BYTES)
    return fail(TJ_ERR_UNSUPPORTED,
                "batch=%d seq_len=%d needs %zu bytes of scratch; tj_forward_noalloc has %u (use tj_forward "
                "with a caller workspace)",
                B, S, need, (unsigned)TJ_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  TJ_CHECK(noalloc_scratch(&scratch));
  // The array keeps the previous call's contents (possibly for another shape,
  // carved differently); tj_forward expects zero-filled scratch.
  TJ_CUDA(cudaMemsetAsync(scratch, 0, need, static_cast<cudaStream_t>(stream)));
  return tj_forward(m, x, mask, out, B, S, route, scratch, need, stream);
}

int tj_copy_valid_rows(void* dst, const void* src, const int* lengths, int B, int S, size_t row_bytes,
                       void* stream) {
  if (!dst || !src || !lengths || B < 0 || S <= 0 || row_bytes == 0) return fail(TJ_ERR_INVALID, "bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* d = static_cast<uint8_t*>(dst);
  const auto* s = static_cast<const uint8_t*>(src);
  const size_t S_bytes = (size_t)S * row_bytes;
  size_t run0 = 0, run_len = 0;  // pending run of consecutive rows (bytes)
  for (int b = 0; b < B; ++b) {
    const int n = lengths[b];
    if (n < 0 || n > S) return fail(TJ_ERR_INVALID, "lengths[%d] = %d outside [0, %d]", b, n, S);
    const size_t start = (size_t)b * S_bytes, bytes = (size_t)n * row_bytes;
    if (bytes == 0) continue;
    if (run_len > 0 && run0 + run_len == start) {
      run_len += bytes;  // previous sample was full: extend the run
      continue;
    }
    if (run_len > 0) TJ_CUDA(cudaMemcpyAsync(d + run0, s + run0, run_len, cudaMemcpyDefault, st));
    run0 = start;
    run_len = bytes;
  }
  if (run_len > 0) TJ_CUDA(cudaMemcpyAsync(d + run0, s + run0, run_len, cudaMemcpyDefault, st));
  return TJ_OK;
}

int tj_poly_workspace_bytes(int B, int H, int S, int exact_prefix, size_t* bytes) {
  if (!bytes || B <= 0 || H <= 0 || S <= 0) return fail(TJ_ERR_INVALID, "bad arguments");
  if (S % tj::kPolyChunk || exact_prefix % tj::kPolyChunk || exact_prefix < tj::kPolyChunk || exact_prefix >= S)
    return fail(TJ_ERR_UNSUPPORTED, "polynomial route needs seq_len and exact_prefix multiples of 512, 512 <= prefix < seq_len");
  const size_t n_snap = (size_t)(S - exact_prefix) / tj::kPolyChunk;
  *bytes = align_up(sizeof(tj::PolyCtl), 256) + 2 * (size_t)B * H * n_snap * tj::kPolyN * tj::kPolyFeat +
           2 * (size_t)B * H * 64 * S;  // snapshots, then K^T
  return TJ_OK;
}

int tj_poly_attention_f16(const void* q, const void* k, const void* v, void* ctx, const int* lengths, int B, int H,
                          int S, int exact_prefix, void* ws, size_t ws_bytes, int* err, void* stream) {
  if (!q || !k || !v || !ctx || !lengths || !ws || !err) return fail(TJ_ERR_INVALID, "null argument");
  size_t need = 0;
  TJ_CHECK(tj_poly_workspace_bytes(B, H, S, exact_prefix, &need));
  if (ws_bytes < need) return fail(TJ_ERR_INVALID, "workspace %zu bytes < required %zu", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return fail(TJ_ERR_INVALID, "workspace not 256-byte aligned");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  auto* ctl = static_cast<tj::PolyCtl*>(ws);
  auto* snap = reinterpret_cast<__half*>(static_cast<uint8_t*>(ws) + align_up(sizeof(tj::PolyCtl), 256));
  __half* kt = snap + (size_t)B * H * ((S - exact_prefix) / tj::kPolyChunk) * tj::kPolyN * tj::kPolyFeat;
  tj::AttnParams ap{};
  ap.lengths = lengths; ap.mask = nullptr; ap.general = nullptr; ap.ctx = static_cast<__half*>(ctx);
  ap.S = S; ap.H = H; ap.d_model = H * 64; ap.causal = 1;
  ap.scale_log2 = (float)(0.125 * 1.4426950408889634);
  ap.err = err;
  ap.q_pos0 = 0;
  ap.kv_shard = S;
  ap.kv_shards = 1;
  ap.B = B;
  return launch_poly_route(static_cast<const __half*>(q), static_cast<const __half*>(k),
                           static_cast<const __half*>(v), static_cast<__half*>(ctx), lengths, B, H, S, H * 64,
                           exact_prefix, ctl, snap, kt, nullptr, ap, static_cast<cudaStream_t>(stream));
}

int tj_profile_begin(TjModel* m, int max_launches) {
  if (!m || max_launches <= 0) return fail(TJ_ERR_INVALID, "bad profile arguments");
  if ((int)m->prof_cls.size() < max_launches) {
    const size_t have = m->prof_ev.size();
    m->prof_ev.resize(2 * (size_t)max_launches);
    for (size_t i = have; i < m->prof_ev.size(); ++i) TJ_CUDA(cudaEventCreate(&m->prof_ev[i]));
    m->prof_cls.resize(max_launches);
  }
  m->prof_max = max_launches;
  m->prof_n = 0;
  m->prof_on = true;
  return TJ_OK;
}

int tj_profile_end(TjModel* m, double* ms, long long* counts) {
  if (!m || !ms || !counts) return fail(TJ_ERR_INVALID, "null argument");
  for (int i = 0; i < TJ_K_COUNT; ++i) { ms[i] = 0.0; counts[i] = 0; }
  m->prof_on = false;
  for (int i = 0; i < m->prof_n; ++i) {
    TJ_CUDA(cudaEventSynchronize(m->prof_ev[2 * i + 1]));
    float t = 0.f;
    TJ_CUDA(cudaEventElapsedTime(&t, m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
    ms[m->prof_cls[i]] += t;
    counts[m->prof_cls[i]] += 1;
  }
  m->prof_n = 0;
  return TJ_OK;
}

int tj_set_wait_limit(unsigned long long ns) {
  const unsigned long long v = ns == 0 ? TJ_WAIT_NS : ns;
  TJ_CUDA(cudaMemcpyToSymbol(tj::g_tj_wait_ns, &v, sizeof(v)));
  return TJ_OK;
}

int tj_set_pdl(int mode) {
  if (mode < -1 || mode > 1) return fail(TJ_ERR_INVALID, "PDL mode %d (need -1, 0 or 1)", mode);
  g_pdl_mode.store(mode, std::memory_order_relaxed);
  return TJ_OK;
}

int tj_wait_selftest(TjModel* m, int* err, void* stream) {
  int* word = m != nullptr ? m->err : err;
  if (word == nullptr) return fail(TJ_ERR_INVALID, "need a model or an error word");
  tj::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(word);
  TJ_CUDA(cudaGetLastError());
  return TJ_OK;
}

int tj_profile_collect(TjModel* m, double* ms, long long* counts) {
  if (!m || !ms || !counts) return fail(TJ_ERR_INVALID, "null argument");
  for (int i = 0; i < m->prof_n; ++i) {
    TJ_CUDA(cudaEventSynchronize(m->prof_ev[2 * i + 1]));
    float t = 0.f;
    TJ_CUDA(cudaEventElapsedTime(&t, m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
    ms[m->prof_cls[i]] += t;
    counts[m->prof_cls[i]] += 1;
  }
  return TJ_OK;
}

int tj_launch_count(TjModel* m, long long* count) {
  if (!m || !count) return fail(TJ_ERR_INVALID, "null argument");
  *count = m->launches;
  return TJ_OK;
}

// ------------------------------------------------------------------ building blocks
int tj_prepare_mask(const uint8_t* mask, int B, int S, int* lengths, uint8_t* general, int* tile_list, int* n_live,
                    uint8_t* tile_live, void* stream) {
  if (!lengths || !general || !tile_list || !n_live || !tile_live) return fail(TJ_ERR_INVALID, "null argument");
  if (B <= 0 || S <= 0) return fail(TJ_ERR_INVALID, "batch and seq_len must be positive");
  return launch_prepare(mask, B, S, lengths, general, tile_list, n_live, tile_live, nullptr, nullptr, nullptr,
                        nullptr, static_cast<cudaStream_t>(stream));
}

int tj_layernorm(const float* x, const float* g, const float* b, int B, int S, int d, float eps, void* out,
                 int out_fp16, const int* lengths, const uint8_t* mask, const uint8_t* tile_live, void* stream) {
  if (!x || !g || !b || !out || !lengths || !tile_live) return fail(TJ_ERR_INVALID, "null argument");
  tj::RowValidity rv{lengths, mask, S, (long long)B * S, nullptr};
  return launch_layernorm(x, g, b, out, out_fp16 != 0, out_fp16 == 0, d, eps, rv, tile_live,
                          static_cast<cudaStream_t>(stream));
}

int tj_gemm_f16(const void* a, const void* wgt, const float* bias, int B, int S, int n, int k, int epilogue, void* out,
                const float* resid, void* q, void* kk, void* v, int heads, const int* tile_list, const int* n_live,
                const int* lengths, const uint8_t* mask, int* err, void* stream) {
  if (!a || !wgt || !bias || !tile_list || !n_live || !lengths || !err) return fail(TJ_ERR_INVALID, "null argument");
  if (n % 32 || k % 8) return fail(TJ_ERR_UNSUPPORTED, "need n %% 32 == 0 and k %% 8 == 0");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  tj::GemmParams p{};
  p.M = B * S; p.N = n; p.K = k; p.seq = S;
  p.lengths = lengths; p.mask = mask; p.tile_list = tile_list; p.n_live = n_live; p.bias = bias; p.err = err;
  if (epilogue == TJ_EPI_QKV) {
    if (!q || !kk || !v || heads <= 0 || n % 3 || (n / 3) % heads) return fail(TJ_ERR_INVALID, "bad QKV arguments");
    p.q = static_cast<__half*>(q); p.k = static_cast<__half*>(kk); p.v = static_cast<__half*>(v);
    p.heads = heads; p.d_model = n / 3; p.head_dim = p.d_model / heads;
    if (p.head_dim % 32) return fail(TJ_ERR_UNSUPPORTED, "head_dim must be a multiple of 32");
  } else if (epilogue == TJ_EPI_RESID) {
    if (!out || !resid) return fail(TJ_ERR_INVALID, "null out/resid");
    p.out32 = static_cast<float*>(out); p.resid = resid;
  } else {
    if (!out) return fail(TJ_ERR_INVALID, "null out");
    p.out16 = static_cast<__half*>(out);
  }
  return launch_gemm_epi(epilogue, a, wgt, p, di.sms, static_cast<cudaStream_t>(stream));
}

int tj_attention_f16(const void* q, const void* k, const void* v, void* ctx, int B, int H, int S, int hd, int causal,
                     const int* lengths, const uint8_t* mask, const uint8_t* general, int* err, int* sched,
                     void* stream) {
  if (!q || !k || !v || !ctx || !lengths || !general || !err) return fail(TJ_ERR_INVALID, "null argument");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  tj::AttnParams p{};
  p.lengths = lengths; p.mask = mask; p.general = general; p.ctx = static_cast<__half*>(ctx);
  p.S = S; p.H = H; p.d_model = H * hd; p.causal = causal ? 1 : 0;
  p.scale_log2 = (float)(1.0 / std::sqrt((double)hd) * 1.4426950408889634);
  p.err = err;
  p.q_pos0 = 0;
  p.kv_shard = S;
  p.kv_shards = 1;
  p.B = B;
  p.sched = sched;
  return launch_attention(q, k, v, hd, p, B, static_cast<cudaStream_t>(stream));
}

int tj_attention_shard_f16(const void* q, const void* k_all, const void* v_all, void* ctx, int B, int H, int S_loc,
                           int hd, const int* lengths, const uint8_t* general, int* err, int* sched, int rank,
                           int world, int layout, void* stream) {
  if (!q || !k_all || !v_all || !ctx || !lengths || !general || !err) return fail(TJ_ERR_INVALID, "null argument");
  if (world <= 0 || rank < 0 || rank >= world) return fail(TJ_ERR_INVALID, "rank %d of %d", rank, world);
  if (layout != TJ_SHARD_CONTIGUOUS && layout != TJ_SHARD_ZIGZAG) return fail(TJ_ERR_INVALID, "unknown layout %d", layout);
  if (S_loc <= 0 || S_loc % (layout == TJ_SHARD_ZIGZAG ? 512 : 128) != 0)
    return fail(TJ_ERR_UNSUPPORTED, "seq_local %d must be a multiple of %d", S_loc, layout == TJ_SHARD_ZIGZAG ? 512 : 128);
  tj::AttnParams p{};
  p.lengths = lengths; p.mask = nullptr; p.general = general; p.ctx = static_cast<__half*>(ctx);
  p.S = S_loc; p.H = H; p.d_model = H * hd; p.causal = 1;
  p.scale_log2 = (float)(1.0 / std::sqrt((double)hd) * 1.4426950408889634);
  p.err = err;
  p.kv_shard = S_loc;
  p.kv_shards = world;
  if (layout == TJ_SHARD_ZIGZAG) {
    p.zz_chunk = S_loc / 2;
    p.q_pos0 = rank * p.zz_chunk;
    p.q_pos1 = (2 * world - 1 - rank) * p.zz_chunk;
  } else {
    p.q_pos0 = rank * S_loc;
  }
  p.B = B;
  p.sched = sched;
  return launch_attention(q, k_all, v_all, hd, p, B, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------------ sequence-sharded forward (NCCL)
#include "tj_nccl.cuh"

struct TjComm {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int world = 1;
  int timeout_ms = 60000;
  bool broken = false;
  // Exchange stream of the polynomial route: the head groups' state
  // all-gathers and fix-ups run here under the next groups' update kernels.
  cudaStream_t side = nullptr;
  std::vector<cudaEvent_t> events;
};

namespace {

int nccl_check(TjComm* c, ncclResult_t r, const char* what) {
  if (r == ncclInProgress) r = tj::nccl_settle(c->comm, c->timeout_ms);
  if (r == ncclSuccess) return TJ_OK;
  c->broken = true;
  tj::nccl().CommAbort(c->comm);
  c->comm = nullptr;
  return fail(TJ_ERR_NCCL, "%s: %s", what,
              r == ncclInProgress ? "timed out (peer missing?); communicator aborted" : tj::nccl().GetErrorString(r));
}

struct ShardWorkspace {
  Workspace base;
  tj::PolyCtl* ctl;
  __half* snap;
  __half* kt;       // [B][H][64][S_loc]: this shard's K transposed
  float* total;     // [B*H][80][4224] fp32: this shard's state
  float* gathered;  // [world][B*H][80][4224]
  __half* kg;       // [world][B][H][S_loc][64]: every shard's K (exact route)
  __half* vg;
};

// Head groups the sequence-sharded polynomial route pipelines its state exchange over.
constexpr int kShardExchangeGroups = 4;

bool shard_poly_eligible(const TjConfig& c, int S_loc, int world, int route) {
  if (route == TJ_ROUTE_EXACT || !c.causal || c.d_model / c.num_heads != 64) return false;
  if (S_loc % tj::kPolyChunk != 0 || S_loc <= kPolyExactPrefix) return false;
  return route == TJ_ROUTE_POLY || (long long)S_loc * world >= kPolyAutoMinSeq;
}

size_t carve_shard(const TjConfig& c, int B, int S_loc, int world, int route, uint8_t* base, ShardWorkspace* w) {
  Workspace bw;
  size_t off = carve(c, B, S_loc, TJ_ROUTE_EXACT, base, &bw);
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  ShardWorkspace t{};
  t.base = bw;
  const size_t BH = (size_t)B * c.num_heads;
  if (shard_poly_eligible(c, S_loc, world, route)) {
    const size_t state = BH * tj::kPolyN * tj::kPolyFeat;
    t.ctl = reinterpret_cast<tj::PolyCtl*>(take(sizeof(tj::PolyCtl)));
    t.snap = reinterpret_cast<__half*>(take(2 * BH * (S_loc / tj::kPolyChunk) * tj::kPolyN * tj::kPolyFeat));
    t.kt = reinterpret_cast<__half*>(take(2 * BH * 64 * (size_t)S_loc));
    t.total = reinterpret_cast<float*>(take(4 * state));
    t.gathered = reinterpret_cast<float*>(take(4 * state * world));
  }
  const size_t kv = (size_t)B * c.num_heads * S_loc * (c.d_model / c.num_heads);
  t.kg = reinterpret_cast<__half*>(take(2 * kv * world));
  t.vg = reinterpret_cast<__half*>(take(2 * kv * world));
  if (w) *w = t;
  return off;
}

__global__ void fill_int_kernel(int* dst, int n, int value) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = value;
}

// Attention of one layer on a sequence shard: guarded polynomial route with a
// state exchange, or exact flash over all-gathered K/V.
int shard_attention(TjModel* m, TjComm* cm, ShardWorkspace& w, int layer, int B, int S_loc, int route, int layout,
                    const tj::AttnParams& ap0, cudaStream_t st) {
  const TjConfig& c = m->cfg;
  const int H = c.num_heads, hd = c.d_model / H, d = c.d_model;
  const int world = cm->world, rank = cm->rank;
  const int S_total = S_loc * world;
  auto& nc = tj::nccl();
  bool admit = false;
  if (w.ctl != nullptr) {
    tj::PolyParams pp{};
    pp.q = w.base.q; pp.k = w.base.k; pp.v = w.base.v; pp.ctx = w.base.act; pp.snap = w.snap; pp.kt = w.kt;
    pp.ctl = w.ctl;
    pp.lengths = w.base.lengths;
    pp.B = B; pp.H = H; pp.S = S_loc; pp.d_model = d;
    pp.prefix_chunks = rank == 0 ? kPolyExactPrefix / tj::kPolyChunk : 0;
    pp.scale = 0.125f;
    pp.err = m->err;
    pp.S_total = S_total;
    pp.t_before = (float)rank * (float)S_loc;
    pp.total = w.total;
    pp.all_chunks = 1;
    const long long key[3] = {B, S_loc, world};
    if (std::memcmp(key, m->shard_key, sizeof(key)) != 0) {  // new shard shape: evaluate every layer again
      std::memcpy(m->shard_key, key, sizeof(key));
      m->shard_route.assign(c.num_layers, -1);
    }
    if (m->shard_route[layer] < 0) {
      // guard over every shard's sample, decided identically everywhere; the
      // host needs the verdict (the exchange depends on the route), so this
      // first evaluation reads it back once and caches it for the layer
      TJ_CUDA(cudaMemsetAsync(w.ctl, 0, sizeof(tj::PolyCtl), st));
      tj::poly_guard_kernel<<<dim3(tj::kPolySample / 64, B * H), 256, 0, st>>>(pp);
      TJ_CUDA(cudaGetLastError());
      TJ_CHECK(nccl_check(cm, nc.AllReduce(&w.ctl->sum, &w.ctl->sum, 2, ncclFloat64, ncclSum, cm->comm, st), "guard sum"));
      TJ_CHECK(nccl_check(cm, nc.AllReduce(&w.ctl->maxv, &w.ctl->maxv, 1, ncclFloat64, ncclMax, cm->comm, st), "guard max"));
      tj::PolyParams pf = pp;
      pf.guard_shards = world;  // the pooled sample covers every shard
      tj::poly_guard_finalize<<<1, 1, 0, st>>>(pf);
      TJ_CUDA(cudaGetLastError());
      int flag = 0;
      TJ_CUDA(cudaMemcpyAsync(&flag, &w.ctl->admit, sizeof(int), cudaMemcpyDeviceToHost, st));
      TJ_CUDA(cudaStreamSynchronize(st));
      TJ_CUDA(cudaMemcpyAsync(m->shard_ctl + layer, w.ctl, sizeof(tj::PolyCtl), cudaMemcpyDeviceToDevice, st));
      m->shard_route[layer] = flag != 0 ? 1 : 0;
    } else {
      // cached verdict and coefficients: no guard kernels, no host synchronisation
      TJ_CUDA(cudaMemcpyAsync(w.ctl, m->shard_ctl + layer, sizeof(tj::PolyCtl), cudaMemcpyDeviceToDevice, st));
    }
    admit = m->shard_route[layer] != 0;
    if (admit) {
      const int n_chunks = S_loc / tj::kPolyChunk;
      const uint64_t rows = (uint64_t)B * H * S_loc;
      CUtensorMap tq, tk, tv, tsn;
      TJ_CHECK(make_map_f16(&tq, w.base.q, rows, 64, 128, 64, 128));
      TJ_CHECK(make_map_f16(&tk, w.base.k, rows, 64, 128, 64, 128));
      TJ_CHECK(make_map_f16(&tv, w.base.v, rows, 64, 128, 64, 128));
      const uint64_t snap_rows = (uint64_t)B * H * (n_chunks - pp.prefix_chunks) * tj::kPolyN;
      TJ_CHECK(make_map_f16(&tsn, w.snap, snap_rows, tj::kPolyFeat, tj::kPolyN, 64, 128));
      TJ_CUDA(cudaFuncSetAttribute(tj::poly_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tj::kUpdSmem));
      TJ_CUDA(cudaFuncSetAttribute(tj::poly_apply_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tj::kAppSmem));
      // The state exchange is pipelined over groups of heads: group g's
      // update kernel runs on the compute stream, then its all-gather and
      // fix-up on the exchange stream while groups g+1.. update; each group's
      // apply waits only for its own fix-up.  Only the last group's exchange
      // is exposed.  Every rank issues the same collectives in the same order.
      const int BH = B * H;
      const int groups = std::min(kShardExchangeGroups, BH);
      const int G = (BH + groups - 1) / groups;
      const size_t per = (size_t)tj::kPolyN * tj::kPolyFeat;
      if (cm->side == nullptr) TJ_CUDA(cudaStreamCreateWithFlags(&cm->side, cudaStreamNonBlocking));
      while ((int)cm->events.size() < 2 * groups) {
        cudaEvent_t e;
        TJ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        cm->events.push_back(e);
      }
      TJ_CHECK(timed_launch(m, TJ_K_POLY, 1, st, [&]() -> int {
        tj::poly_k_transpose_kernel<<<dim3(pp.S / 64, BH), 256, 0, st>>>(pp.k, pp.kt, pp.S);
        TJ_CUDA(cudaGetLastError());
        return TJ_OK;
      }));
      CUtensorMap tkt;
      TJ_CHECK(make_map_f16(&tkt, pp.kt, (uint64_t)BH * 64, (uint64_t)pp.S, 64, 64, 128));
      for (int g = 0; g < groups; ++g) {
        tj::PolyParams pg = pp;
        pg.bh0 = g * G;
        const int n = std::min(G, BH - pg.bh0);
        if (n <= 0) break;
        TJ_CHECK(timed_launch(m, TJ_K_POLY, 1, st, [&]() -> int {
          tj::poly_update_kernel<<<dim3(tj::kPolyFeatBlocks, n), 192, tj::kUpdSmem, st>>>(tkt, tv, pg);
          TJ_CUDA(cudaGetLastError());
          return TJ_OK;
        }));
        TJ_CUDA(cudaEventRecord(cm->events[2 * g], st));
        TJ_CUDA(cudaStreamWaitEvent(cm->side, cm->events[2 * g], 0));
        float* gath = w.gathered + (size_t)pg.bh0 * per * world;
        TJ_CHECK(nccl_check(cm, nc.AllGather(w.total + (size_t)pg.bh0 * per, gath, (size_t)n * per, ncclFloat32,
                                             cm->comm, cm->side), "state all-gather"));
        if (rank > 0) {
          tj::poly_fixup_kernel<<<1184, 256, 0, cm->side>>>(gath, rank, n, pg.bh0, w.snap,
                                                            n_chunks - pp.prefix_chunks, pp.prefix_chunks,
                                                            pp.t_before);
          TJ_CUDA(cudaGetLastError());
        }
        TJ_CUDA(cudaEventRecord(cm->events[2 * g + 1], cm->side));
      }
      for (int g = 0; g < groups; ++g) {
        tj::PolyParams pg = pp;
        pg.bh0 = g * G;
        const int n = std::min(G, BH - pg.bh0);
        if (n <= 0) break;
        TJ_CUDA(cudaStreamWaitEvent(st, cm->events[2 * g + 1], 0));
        TJ_CHECK(timed_launch(m, TJ_K_POLY, 1, st, [&]() -> int {
          tj::poly_apply_kernel<<<dim3((n_chunks - pp.prefix_chunks) * 4, n), tj::kAppThreads, tj::kAppSmem, st>>>(
              tq, tk, tv, tsn, pg);
          TJ_CUDA(cudaGetLastError());
          return TJ_OK;
        }));
      }
      if (rank == 0) {  // exact prefix: every key it needs is local
        tj::AttnParams ap = ap0;
        ap.poly_admit = &w.ctl->admit;
        ap.exact_pairs = kPolyExactPrefix / 256;
        ap.q_pos0 = 0;
        ap.kv_shard = S_loc;
        ap.kv_shards = 1;
        TJ_CHECK(timed_launch(m, TJ_K_ATTN, 1, st, [&] { return launch_attention(w.base.q, w.base.k, w.base.v, 64,
                                                                                  ap, B, st); }));
      }
      return TJ_OK;
    }
  }
  // exact route: gather every shard's K and V, then local queries at their global positions
  const size_t kv = (size_t)B * H * S_loc * hd;
  TJ_CHECK(nccl_check(cm, nc.AllGather(w.base.k, w.kg, kv, ncclFloat16, cm->comm, st), "K all-gather"));
  TJ_CHECK(nccl_check(cm, nc.AllGather(w.base.v, w.vg, kv, ncclFloat16, cm->comm, st), "V all-gather"));
  tj::AttnParams ap = ap0;
  ap.poly_admit = nullptr;
  ap.kv_shard = S_loc;
  ap.kv_shards = world;
  if (layout == TJ_SHARD_ZIGZAG) {  // chunks rank and 2*world-1-rank of S_loc/2 tokens
    ap.zz_chunk = S_loc / 2;
    ap.q_pos0 = rank * ap.zz_chunk;
    ap.q_pos1 = (2 * world - 1 - rank) * ap.zz_chunk;
  } else {
    ap.q_pos0 = rank * S_loc;
  }
  return timed_launch(m, TJ_K_ATTN, 1, st, [&] { return launch_attention(w.base.q, w.kg, w.vg, hd, ap, B, st); });
}

}  // namespace

extern "C" {

int tj_nccl_unique_id(void* id_out) {
  if (!id_out) return fail(TJ_ERR_INVALID, "null argument");
  auto& nc = tj::nccl();
  if (!nc.ok) return fail(TJ_ERR_NCCL, "NCCL unavailable: %s", nc.why);
  ncclUniqueId id;
  const ncclResult_t r = nc.GetUniqueId(&id);
  if (r != ncclSuccess) return fail(TJ_ERR_NCCL, "ncclGetUniqueId: %s", nc.GetErrorString(r));
  std::memcpy(id_out, &id, sizeof(id));
  return TJ_OK;
}

int tj_comm_create(const void* id, int rank, int world, int timeout_ms, TjComm** out) {
  if (!id || !out || world <= 0 || rank < 0 || rank >= world) return fail(TJ_ERR_INVALID, "bad communicator arguments");
  *out = nullptr;
  auto& nc = tj::nccl();
  if (!nc.ok) return fail(TJ_ERR_NCCL, "NCCL unavailable: %s", nc.why);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  auto* c = new TjComm();
  c->rank = rank;
  c->world = world;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  ncclResult_t r = nc.CommInitRankConfig(&c->comm, world, uid, rank, &cfg);
  if (r == ncclInProgress || r == ncclSuccess) r = tj::nccl_settle(c->comm, c->timeout_ms);
  if (r != ncclSuccess) {
    if (c->comm) nc.CommAbort(c->comm);
    delete c;
    return fail(TJ_ERR_NCCL, "ncclCommInitRankConfig: %s",
                r == ncclInProgress ? "timed out waiting for the other ranks" : nc.GetErrorString(r));
  }
  *out = c;
  return TJ_OK;
}

int tj_comm_destroy(TjComm* c) {
  if (!c) return TJ_OK;
  for (cudaEvent_t e : c->events) cudaEventDestroy(e);
  if (c->side) cudaStreamDestroy(c->side);
  if (c->comm) {
    if (c->broken) tj::nccl().CommAbort(c->comm);
    else tj::nccl().CommDestroy(c->comm);
  }
  delete c;
  return TJ_OK;
}

int tj_seqshard_route(const TjModel* m, int layer, int* route) {
  if (!m || !route) return fail(TJ_ERR_INVALID, "null argument");
  if (layer < 0 || layer >= m->cfg.num_layers) return fail(TJ_ERR_INVALID, "layer %d out of range", layer);
  *route = m->shard_route[layer];
  return TJ_OK;
}

int tj_workspace_bytes_seqshard(const TjModel* m, const TjComm* c, int B, int S_loc, int route, size_t* bytes) {
  if (!m || !c || !bytes || B <= 0 || S_loc <= 0) return fail(TJ_ERR_INVALID, "bad arguments");
  *bytes = carve_shard(m->cfg, B, S_loc, c->world, route, nullptr, nullptr);
  return TJ_OK;
}

int tj_forward_seqshard(TjModel* m, TjComm* cm, const float* x, float* out, int B, int S_loc, int route, int layout,
                        void* ws, size_t ws_bytes, void* stream) {
  if (!m || !cm || !x || !out || !ws) return fail(TJ_ERR_INVALID, "null argument");
  if (cm->broken || !cm->comm) return fail(TJ_ERR_NCCL, "communicator is broken");
  if (B <= 0 || S_loc <= 0 || S_loc % 128) return fail(TJ_ERR_UNSUPPORTED, "seq_len per shard must be a multiple of 128");
  if (x == out) return fail(TJ_ERR_INVALID, "x and out must not alias");
  if (!m->cfg.causal) return fail(TJ_ERR_UNSUPPORTED, "sequence sharding needs causal attention");
  if (layout != TJ_SHARD_CONTIGUOUS && layout != TJ_SHARD_ZIGZAG) return fail(TJ_ERR_INVALID, "unknown layout %d", layout);
  if (layout == TJ_SHARD_ZIGZAG && route != TJ_ROUTE_EXACT)
    return fail(TJ_ERR_UNSUPPORTED, "the zig-zag layout balances the exact route; pass TJ_ROUTE_EXACT");
  if (layout == TJ_SHARD_ZIGZAG && S_loc % 512 != 0)
    return fail(TJ_ERR_UNSUPPORTED, "zig-zag sharding needs seq_local a multiple of 512 (two 256-aligned chunks)");
  const TjConfig& c = m->cfg;
  const size_t need = carve_shard(c, B, S_loc, cm->world, route, nullptr, nullptr);
  if (ws_bytes < need) return fail(TJ_ERR_INVALID, "workspace %zu bytes < required %zu", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return fail(TJ_ERR_INVALID, "workspace not 256-byte aligned");
  DeviceInfo di;
  TJ_CHECK(device_info(&di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ShardWorkspace w;
  carve_shard(c, B, S_loc, cm->world, route, static_cast<uint8_t*>(ws), &w);
  const int d = c.d_model, H = c.num_heads, hd = d / H, F = c.ffn_dim;
  const int M = B * S_loc;
  const int S_total = S_loc * cm->world;
  // unpadded sequences of S_total tokens; every local row is valid
  TJ_CHECK(timed_launch(m, TJ_K_PREP, 2, st, [&]() -> int {
    fill_int_kernel<<<(B + 255) / 256, 256, 0, st>>>(w.base.lengths, B, S_total);
    TJ_CUDA(cudaGetLastError());
    TJ_CUDA(cudaMemsetAsync(w.base.general, 0, B, st));
    TJ_CUDA(cudaMemsetAsync(w.base.sched, 0, 2 * sizeof(int), st));
    tj::prep_tiles_kernel<<<1, 1024, 0, st>>>(w.base.lengths, B, S_loc, w.base.tile_list, w.base.n_live,
                                              w.base.tile_live);
    TJ_CUDA(cudaGetLastError());
    return TJ_OK;
  }));
  tj::RowValidity rv{w.base.lengths, nullptr, S_loc, (long long)M, nullptr};
  tj::GemmParams gp{};
  gp.M = M; gp.seq = S_loc; gp.lengths = w.base.lengths; gp.mask = nullptr;
  gp.tile_list = w.base.tile_list; gp.n_live = w.base.n_live;
  gp.q = w.base.q; gp.k = w.base.k; gp.v = w.base.v;
  gp.heads = H; gp.head_dim = hd; gp.d_model = d; gp.err = m->err;
  tj::AttnParams ap{};
  ap.lengths = w.base.lengths; ap.mask = nullptr; ap.general = w.base.general; ap.ctx = w.base.act;
  ap.S = S_loc; ap.H = H; ap.d_model = d; ap.causal = 1;
  ap.scale_log2 = (float)(1.0 / std::sqrt((double)hd) * 1.4426950408889634);
  ap.err = m->err; ap.B = B; ap.kv_shard = S_loc; ap.kv_shards = 1; ap.q_pos0 = 0; ap.sched = w.base.sched;
  const float eps = c.layer_norm_eps;
  const float* resid_in = x;
  for (int l = 0; l < c.num_layers; ++l) {
    const TjLayerPacked& L = m->layers[l];
    TJ_CHECK(timed_launch(m, TJ_K_LN, 1, st, [&] {
      return launch_layernorm(resid_in, L.ln1_g, L.ln1_b, w.base.act, true, false, d, eps, rv, w.base.tile_live, st);
    }));
    gp.N = 3 * d; gp.K = d; gp.bias = L.bqkv;
    TJ_CHECK(timed_launch(m, TJ_K_QKV, 1, st, [&] { return launch_gemm_epi(tj::kEpiQKV, w.base.act, L.wqkv, gp, di.sms, st); }));
    TJ_CHECK(shard_attention(m, cm, w, l, B, S_loc, route, layout, ap, st));
    gp.N = d; gp.K = d; gp.bias = L.bo; gp.out32 = out; gp.resid = resid_in;
    TJ_CHECK(timed_launch(m, TJ_K_OUT, 1, st, [&] { return launch_gemm_epi(tj::kEpiResid, w.base.act, L.wo, gp, di.sms, st); }));
    TJ_CHECK(timed_launch(m, TJ_K_LN, 1, st, [&] {
      return launch_layernorm(out, L.ln2_g, L.ln2_b, w.base.act, true, false, d, eps, rv, w.base.tile_live, st);
    }));
    gp.N = F; gp.K = d; gp.bias = L.b1; gp.out16 = w.base.ff;
    TJ_CHECK(timed_launch(m, TJ_K_FFN_IN, 1, st, [&] { return launch_gemm_epi(tj::kEpiGelu, w.base.act, L.w1, gp, di.sms, st); }));
    gp.N = d; gp.K = F; gp.bias = L.b2; gp.out32 = out; gp.resid = out;
    TJ_CHECK(timed_launch(m, TJ_K_FFN_OUT, 1, st, [&] { return launch_gemm_epi(tj::kEpiResid, w.base.ff, L.w2, gp, di.sms, st); }));
    resid_in = out;
  }
  TJ_CHECK(timed_launch(m, TJ_K_LN_FINAL, 1, st, [&] {
    return launch_layernorm(out, m->final_g, m->final_b, out, false, true, d, eps, rv, w.base.tile_live, st);
  }));
  return TJ_OK;
}

}  // extern "C"
