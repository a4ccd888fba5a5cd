// Guarded degree-2 polynomial (Hermite/Taylor-exp) causal linear attention
// for long unpadded sequences, head_dim 64.
//
// Algorithm (the reference's poly_linear_attention): keys in EARLIER 512-token
// chunks are weighted by w(s) = c0 + c1 s + c2 s^2 (s = q.k * scale), keys in
// the SAME chunk by the exact exp(s) with the causal triangle, queries in the
// first `exact_prefix` tokens by exact softmax (the flash kernel).
//
// B200 formulation.  With the 4224-wide feature maps
//     phi_k(k) = [ scale k_i k_j (4096) | sqrt(scale) k_i (64) | 1 | 0 x 63 ]
//     phi_q(q) = [ c2 scale q_i q_j     | c1 sqrt(scale) q_i   | c0 | 0 ... ]
// phi_q(q) . phi_k(k) = w(q.k * scale), so for every query of chunk c
//     [num | den] = phi_q(q) @ S_c + sum_{j in chunk, j <= i} exp(s_ij) [v_j | 1]
// where S_c = sum over keys before chunk c of phi_k(k)^T [v | 1]  (4224 x 65).
// The snapshots keep the denominator as column 64 of S_c, so in the apply
// kernel numerator and denominator of all three polynomial orders come out of
// one N = 80 tensor-core accumulation; the update kernel forms that column
// and the exact diagonal block's denominator as per-thread FP32 row sums.
//
//   poly_guard_kernel/poly_guard_finalize  score std (sigma) and max |s| over a
//       fixed strided sample of 512 rows per head -> PolyCtl (admit flag and
//       Hermite coefficients), on the device: no host synchronisation.  Every
//       poly kernel exits at once unless admitted; the flash kernel then covers
//       the whole sequence instead of only the exact prefix.
//   poly_k_transpose_kernel  K^T per head, so feature rows are contiguous.
//   poly_update_kernel  one CTA per (128-feature block, head): per 128-token
//       sub-chunk each thread forms one feature row (over the tokens) and
//       stores it to its TMEM lane, the tensor core accumulates
//       phi_k^T [v | 1] (A from TMEM) in TMEM (double-buffered per chunk); the
//       running state stays in registers (fp32) and after every chunk the
//       MEAN state S_c / (512 c) is stored as fp16 (keeps the fp16 snapshot in
//       range however long the sequence).
//   poly_apply_kernel   one CTA per (128-query block, head): phi_q(q) @ S_c
//       over 33 feature blocks (K = 4224; phi_q rows written to TMEM as the A
//       operand) plus the exact-exp diagonal block, then
//       out = (512c * inter + diag)[:64] / (512c * inter + diag)[64].
#pragma once
#include "tj_common.cuh"

namespace tj {

constexpr int kPolyChunk = 512;
constexpr int kPolyFeat = 4224;       // 4096 + 64 + 1, padded to 33 blocks of 128
constexpr int kPolyFeatBlocks = 33;
constexpr int kPolyN = 80;            // 64 numerator + 1 denominator, padded to N % 16 == 0
constexpr int kPolySample = 512;      // rows per head in the guard's sample
constexpr float kPolySigmaCeiling = 0.40f;
constexpr float kPolyMaxScore = 10.0f;  // exp(s) of the diagonal block stays < fp16 max

struct PolyCtl {
  int admit;  // 1: polynomial route, 0: exact route
  float c0, c1, c2;
  float sigma;
  float max_abs;
  double sum, sumsq, maxv;  // guard accumulators
  int sched[2];             // work scheduler of the exact-prefix flash launch
};

struct PolyParams {
  const __half* q;  // [B, H, S, 64]
  const __half* k;
  const __half* v;
  __half* ctx;      // [B*S, d_model]
  __half* kt;       // [B, H, 64, S] fp16: K transposed (the update kernel's feature rows)
  __half* snap;     // [B*H][n_snap][80][4224] fp16 mean states
  PolyCtl* ctl;
  const int* lengths;
  int B, H, S, d_model;
  int prefix_chunks;  // exact prefix / 512 (0 on sequence shards after the first)
  float scale;        // head_dim^-0.5
  int* err;
  // Sequence sharding (unsharded: S_total = S, t_before = 0, total = null,
  // all_chunks = 0): this shard holds global tokens [t_before, t_before + S)
  // of sequences S_total long; the update also runs over the last local
  // chunk and writes the shard's total state (fp32 [B*H][80][4224]).
  int S_total;
  float t_before;
  float* total;
  int all_chunks;
  int guard_shards;  // shards whose guard samples were pooled (all-reduced) before finalize
  // The update and apply kernels cover heads bh0 .. bh0 + gridDim.y - 1 of
  // the B*H (batch, head) pairs (0 for a launch over all of them).
  int bh0;
};

// ------------------------------------------------------------------ guard
// blockIdx.y = b*H + h; blockIdx.x = block of 64 sampled query rows.  The
// sample is the strided row set {floor(r * S / 512) : r < 512} of each head
// (the reference draws 512 rows with a seeded randperm; any fixed spread
// sample estimates the same population spread).  Scores use the fp16 q/k
// the attention consumes, accumulated in fp32.
__global__ void __launch_bounds__(256) poly_guard_kernel(PolyParams p) {
  __shared__ float qs[64][65];
  __shared__ float ks[64][65];
  __shared__ double dred[2][8];
  __shared__ float mred[8];
  const int bh = blockIdx.y;
  const __half* qb = p.q + (size_t)bh * p.S * 64;
  const __half* kb = p.k + (size_t)bh * p.S * 64;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int r = i >> 6, c = i & 63;
    const long long row = (long long)(blockIdx.x * 64 + r) * p.S / kPolySample;
    qs[r][c] = __half2float(qb[row * 64 + c]);
  }
  const int qi = threadIdx.x >> 2;  // query row of this thread
  const int k0 = threadIdx.x & 3;   // keys k0, k0+4, ... of each tile
  double sum = 0.0, sumsq = 0.0;
  float mx = 0.0f;
  for (int kt = 0; kt < kPolySample / 64; ++kt) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
      const int r = i >> 6, c = i & 63;
      const long long row = (long long)(kt * 64 + r) * p.S / kPolySample;
      ks[r][c] = __half2float(kb[row * 64 + c]);
    }
    __syncthreads();
    float s_loc = 0.f, s2_loc = 0.f;
    for (int kk = k0; kk < 64; kk += 4) {
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 64; ++e) dot = fmaf(qs[qi][e], ks[kk][e], dot);
      dot *= p.scale;
      s_loc += dot;
      s2_loc += dot * dot;
      mx = fmaxf(mx, fabsf(dot));
    }
    sum += s_loc;
    sumsq += s2_loc;
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    sumsq += __shfl_xor_sync(0xffffffffu, sumsq, o);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { dred[0][w] = sum; dred[1][w] = sumsq; mred[w] = mx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0, s2 = 0;
    float m = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { s += dred[0][i]; s2 += dred[1][i]; m = fmaxf(m, mred[i]); }
    atomicAdd(&p.ctl->sum, s);
    atomicAdd(&p.ctl->sumsq, s2);
    // non-negative doubles order like their bit patterns
    atomicMax(reinterpret_cast<unsigned long long*>(&p.ctl->maxv), (unsigned long long)__double_as_longlong((double)m));
  }
}

// Single thread: sigma (unbiased std like torch.std), admission, coefficients.
__global__ void poly_guard_finalize(PolyParams p) {
  PolyCtl* c = p.ctl;
  const double n = (double)p.B * p.H * (p.guard_shards > 0 ? p.guard_shards : 1) * kPolySample * kPolySample;
  const double mean = c->sum / n;
  const double var = (c->sumsq - n * mean * mean) / (n - 1.0);
  const float sigma = (float)sqrt(var > 0 ? var : 0.0);
  const float mx = (float)c->maxv;
  bool unpadded = true;
  for (int b = 0; b < p.B; ++b) unpadded = unpadded && (p.lengths[b] == p.S_total);
  const bool ok = isfinite(sigma) && isfinite(mx) && sigma > 0.f && sigma <= kPolySigmaCeiling &&
                  mx <= kPolyMaxScore && unpadded;
  const float g = expf(0.5f * sigma * sigma);
  c->c0 = g * fmaxf(1.0f - 0.5f * sigma * sigma, 1e-3f);
  c->c1 = g;
  c->c2 = 0.5f * g;
  c->sigma = sigma;
  c->max_abs = mx;
  c->admit = ok ? 1 : 0;
}

// ------------------------------------------------------------------ feature rows
// Q, K, V tiles are [128 rows x 64] fp16 with the 128-byte swizzle (16-byte
// chunk c of row r at c ^ (r & 7)); feature maps are formed in registers and
// written to TMEM, where they are the A operand of the tensor-core products.
// Row `row` of a [128 x 64] fp16 tile (128-byte swizzle) as 32 packed halves pairs.
TJ_DEV void load_row_h2(const uint8_t* tile, int row, uint32_t (&h)[32]) {
  const uint8_t* base = tile + row * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(base + ((c ^ (row & 7)) << 4));
    h[4 * c] = w.x; h[4 * c + 1] = w.y; h[4 * c + 2] = w.z; h[4 * c + 3] = w.w;
  }
}

// Elements (i, i+1) (i even) of a row of a [128 x 64] fp16 tile (128B swizzle).
TJ_DEV float2 load_pair(const uint8_t* tile, int row, int i) {
  const uint8_t* a = tile + row * 128 + (((i >> 3) ^ (row & 7)) << 4) + (i & 7) * 2;
  return __half22float2(*reinterpret_cast<const __half2*>(a));
}

// w = coef * h (64 fp16 values as 32 pairs), packed fp16 multiplies.
TJ_DEV void scale_row_h2(const uint32_t (&h)[32], float coef, uint32_t (&w)[32]) {
  const __half2 c2 = __float2half2_rn(coef);
  const uint32_t cw = *reinterpret_cast<const uint32_t*>(&c2);
#pragma unroll
  for (int e = 0; e < 32; ++e) asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w[e]) : "r"(h[e]), "r"(cw));
}

// Chunk c's delta (numerator from TMEM buffer c & 1, denominator `den` summed
// by the thread itself), times the feature row's coefficient (scale,
// sqrt(scale) or 1), -> running fp32 state (registers) -> fp16 MEAN snapshot
// for chunk c+1 (row frow of feature block fb).
TJ_DEV bool update_drain(const PolyParams& p, uint32_t tmem, int quarter, int frow, int fb, int bh, int c,
                         int n_chunks, uint64_t* d_full, uint64_t* d_empty, float coef, float den,
                         float (&state)[65]) {
  const int db = c & 1;
  if (!mbar_wait(d_full + db, (c >> 1) & 1, p.err, kErrPolyWait)) return false;
  tc_fence_after();
  uint32_t r[32];
  const uint32_t a = tmem + ((uint32_t)(quarter * 32) << 16) + db * 128;
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    tmem_ld32(a + part * 32, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) state[part * 32 + i] = fmaf(coef, __uint_as_float(r[i]), state[part * 32 + i]);
  }
  state[64] = fmaf(coef, den, state[64]);
  tc_fence_before();
  mbar_arrive(d_empty + db);
  const int cn = c + 1;
  if (p.total != nullptr && cn == n_chunks) {  // the shard's total state, fp32
    float* dst = p.total + ((size_t)bh * kPolyN) * kPolyFeat + (size_t)fb * 128 + frow;
#pragma unroll
    for (int n = 0; n < kPolyN; ++n) dst[(size_t)n * kPolyFeat] = n < 65 ? state[n] : 0.f;
  }
  if (cn >= p.prefix_chunks && cn < n_chunks) {
    const float inv = 1.0f / (float)(cn * kPolyChunk);
    __half* dst = p.snap +
                  (((size_t)bh * (n_chunks - p.prefix_chunks) + (cn - p.prefix_chunks)) * kPolyN) * kPolyFeat +
                  (size_t)fb * 128 + frow;
#pragma unroll
    for (int n = 0; n < kPolyN; ++n) dst[(size_t)n * kPolyFeat] = __float2half_rn(n < 65 ? state[n] * inv : 0.f);
  }
  return true;
}

// ------------------------------------------------------------------ update
// kt[bh][d][t] = k[bh][t][d]: the update kernel reads feature rows (a key
// dimension over 128 tokens) as contiguous shared-memory rows.
__global__ void __launch_bounds__(256) poly_k_transpose_kernel(const __half* __restrict__ k, __half* __restrict__ kt,
                                                               int S) {
  __shared__ __half tile[64][72];  // [token][dim], 16-byte padded rows
  const int bh = blockIdx.y;
  const int t0 = blockIdx.x * 64;
  const __half* src = k + ((size_t)bh * S + t0) * 64;
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int r = i >> 3, c = (i & 7) * 8;
    *reinterpret_cast<uint4*>(&tile[r][c]) = *reinterpret_cast<const uint4*>(src + (size_t)r * 64 + c);
  }
  __syncthreads();
  __half* dst = kt + (size_t)bh * 64 * S + t0;
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int d = i >> 3, c = (i & 7) * 8;
    __align__(16) __half v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = tile[c + e][d];
    *reinterpret_cast<uint4*>(dst + (size_t)d * S + c) = *reinterpret_cast<const uint4*>(v);
  }
}

// 64 halves (32 pairs) of row `row` of a [64 x 64] fp16 box with the 128-byte swizzle.
TJ_DEV void load_box_row(const uint8_t* box, int row, uint32_t* h) {
  const uint8_t* base = box + row * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(base + ((c ^ (row & 7)) << 4));
    h[4 * c] = w.x; h[4 * c + 1] = w.y; h[4 * c + 2] = w.z; h[4 * c + 3] = w.w;
  }
}

constexpr int kUpdStages = 5;     // K^T / V sub-chunk ring
constexpr int kUpdPhiBufs = 2;    // phi_k sub-chunk tiles, in TMEM
constexpr int kUpdSmem = kUpdStages * 32768 + 1024 + 256;

// One CTA per (128-feature block fb, head).  Thread L of the generator warps
// owns feature row L of the block (TMEM lane L): for fb < 32 the product
// k_{2fb + L/64} * k_{L%64} over the sub-chunk's 128 tokens (packed fp16
// multiplies of two K^T rows), for fb = 32 the linear rows k_L (L < 64), the
// constant row (L = 64) and zeros; its coefficient (scale, sqrt(scale), 1) is
// applied when the chunk's delta is drained.  The rows go straight into TMEM
// as the A operand of phi_k^T V (TS form), so shared memory carries only K^T
// and V; the denominator column phi_k^T 1 is each thread's own row sum (FP32
// adds of the fp16 features), which saves the N = 16 MMA per 16 tokens that a
// ones operand would cost (every tcgen05.mma takes ~100 cycles at N <= 64).
__global__ void __launch_bounds__(192, 1)
    poly_update_kernel(const __grid_constant__ CUtensorMap tmKt, const __grid_constant__ CUtensorMap tmV,
                       const PolyParams p) {
  if (p.ctl->admit == 0 || error_raised(p.err)) return;
  const int fb = blockIdx.x;
  const int bh = p.bh0 + (int)blockIdx.y;
  const int n_chunks = p.S / kPolyChunk;
  // the last chunk's keys feed no later query of this shard (only later shards)
  const int n_sub = (p.all_chunks ? n_chunks : n_chunks - 1) * 4;
  if (n_sub <= 0) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem;                                  // stage: K^T 2 x 8 KB | V 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kUpdStages * 32768);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + kUpdStages;
  uint64_t* phi_full = kv_empty + kUpdStages;
  uint64_t* phi_empty = phi_full + kUpdPhiBufs;
  uint64_t* d_full = phi_empty + kUpdPhiBufs;  // [2] chunk delta ready
  uint64_t* d_empty = d_full + 2;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    // 128 generator threads read each K^T stage (+ the MMA commit for V)
    for (int i = 0; i < kUpdStages; ++i) { mbar_init(kv_full + i, 1); mbar_init(kv_empty + i, 129); }
    for (int i = 0; i < kUpdPhiBufs; ++i) { mbar_init(phi_full + i, 128); mbar_init(phi_empty + i, 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(d_full + i, 1); mbar_init(d_empty + i, 128); }
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: deltas [0, 64) [128, 192) | phi_k [256, 320) [320, 384)
  const uint32_t t_phi = tmem + 256;
  const int row0 = bh * p.S;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmKt);
      tma_prefetch_desc(&tmV);
      for (int u = 0; u < n_sub; ++u) {
        const int st = u % kUpdStages;
        if (!mbar_wait(kv_empty + st, ((u / kUpdStages) & 1) ^ 1, p.err, kErrPolyWait)) break;
        mbar_expect_tx(kv_full + st, 32768);
        tma_load_2d(sKV + st * 32768, &tmKt, kv_full + st, u * 128, bh * 64);
        tma_load_2d(sKV + st * 32768 + 8192, &tmKt, kv_full + st, u * 128 + 64, bh * 64);
        tma_load_2d(sKV + st * 32768 + 16384, &tmV, kv_full + st, 0, row0 + u * 128);
      }
    }
  } else if (warp == 1) {
    {  // the whole warp: every wait agrees in all lanes; tcgen05 issues come from the elected lane
      constexpr uint32_t idesc_v = idesc_f16_f32(128, 64, false, true);   // A from TMEM, B (V) MN-major
      bool ok = true;
      for (int u = 0; u < n_sub && ok; ++u) {
        const int st = u % kUpdStages, pb = u % kUpdPhiBufs;
        const int c = u >> 2, db = c & 1;
        if ((u & 3) == 0 && !mbar_wait_warp(d_empty + db, ((c >> 1) & 1) ^ 1, p.err, kErrPolyWait)) { ok = false; break; }
        if (!mbar_wait_warp(kv_full + st, (u / kUpdStages) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        if (!mbar_wait_warp(phi_full + pb, (u / kUpdPhiBufs) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t phi = t_phi + pb * 64;
        const uint32_t vv = smem_u32(sKV + st * 32768 + 16384);
        const uint32_t d = tmem + db * 128;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // K = 128 tokens, 16 per MMA (8 TMEM columns)
          const uint64_t bv = smem_desc(vv + ks * 2048, 8192, 1024, 128);
          umma_f16_ts_elect(d, phi + ks * 8, bv, idesc_v, ((u & 3) | ks) != 0);
        }
        umma_commit_elect(kv_empty + st);
        umma_commit_elect(phi_empty + pb);
        if ((u & 3) == 3) umma_commit_elect(d_full + db);
      }
    }
  } else {
    // ---------------------------------------------------- phi_k rows + state epilogue
    const int quarter = warp & 3;          // TMEM lanes of this warp
    const int frow = quarter * 32 + lane;  // feature row of this thread (generation and epilogue)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int a = frow >> 6, j = frow & 63;
    const float coef = fb < 32 ? p.scale : (frow < 64 ? sqrtf(p.scale) : 1.0f);
    float state[65];
#pragma unroll
    for (int n = 0; n < 65; ++n) state[n] = 0.f;
    float den_chunk = 0.f, den_prev = 0.f;  // row sums of the chunk being built / awaiting drain
    bool ok = true;
    for (int u = 0; u < n_sub && ok; ++u) {
      const int st = u % kUpdStages, pb = u % kUpdPhiBufs;
      if ((u & 3) == 0) {
        den_prev = den_chunk;
        den_chunk = 0.f;
      }
      if (!mbar_wait(kv_full + st, (u / kUpdStages) & 1, p.err, kErrPolyWait)) { ok = false; break; }
      if (!mbar_wait(phi_empty + pb, ((u / kUpdPhiBufs) & 1) ^ 1, p.err, kErrPolyWait)) { ok = false; break; }
      tc_fence_after();
      const uint8_t* kt_st = sKV + st * 32768;
      float dsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // tokens 64*hh .. +63 -> TMEM columns 32*hh .. +31
        uint32_t w[32];
        if (fb < 32) {
          uint32_t ki[32];
          load_box_row(kt_st + hh * 8192, j, w);
          load_box_row(kt_st + hh * 8192, 2 * fb + a, ki);
#pragma unroll
          for (int e = 0; e < 32; ++e) asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w[e]) : "r"(w[e]), "r"(ki[e]));
        } else if (frow < 64) {
          load_box_row(kt_st + hh * 8192, j, w);
        } else {
          const uint32_t fill = frow == 64 ? 0x3C003C00u : 0u;  // the constant feature: 1 per token
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = fill;
        }
        tmem_st32(t_phi + pb * 64 + hh * 32 + lane_off, w);
#pragma unroll
        for (int e = 0; e < 32; ++e) {  // the row's denominator contribution, FP32
          unsigned short lo, hi;
          asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(w[e]));
          asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(dsum[e & 3]) : "h"(lo), "f"(dsum[e & 3]));
          asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(dsum[e & 3]) : "h"(hi), "f"(dsum[e & 3]));
        }
      }
      den_chunk += (dsum[0] + dsum[1]) + (dsum[2] + dsum[3]);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(phi_full + pb);
      mbar_arrive(kv_empty + st);  // K^T rows read (the MMA commit covers V)
      // drain the previous chunk's delta once this chunk's first sub-chunk is queued
      if ((u & 3) == 0 && u >= 4 &&
          !update_drain(p, tmem, quarter, frow, fb, bh, (u >> 2) - 1, n_chunks, d_full, d_empty, coef, den_prev,
                        state)) {
        ok = false;
        break;
      }
    }
    if (ok)
      update_drain(p, tmem, quarter, frow, fb, bh, (n_sub >> 2) - 1, n_chunks, d_full, d_empty, coef, den_chunk, state);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ apply
constexpr int kAppSnapStages = 6;  // snapshot K-block ring (2 x [80 x 64] fp16 = 20 KB)
constexpr int kAppSnapBytes = 20480;
constexpr int kAppPhiBufs = 2;     // phi_q feature blocks, in TMEM
constexpr int kAppSmem = 16384 /*Q*/ + 2 * 32768 /*diag K,V ring*/ + kAppSnapStages * kAppSnapBytes +
                         1024 + 256;
// warp 0 TMA; warps 1 and 2 issue the feature-block MMAs (even / odd blocks,
// each into its own accumulator: a tcgen05.mma costs its issuing warp ~105
// cycles however small N is, and two issuers halve that chain); warp 1 also
// issues the diagonal block; warps 3..6 phi_q, diagonal exp and epilogue
constexpr int kAppThreads = 224;

__global__ void __launch_bounds__(kAppThreads, 1)
    poly_apply_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmSnap,
                      const PolyParams p) {
  if (p.ctl->admit == 0 || error_raised(p.err)) return;
  const int bh = p.bh0 + (int)blockIdx.y;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int n_chunks = p.S / kPolyChunk;
  const int u = p.prefix_chunks * 4 + (int)blockIdx.x;  // global 128-query block
  const int c = u >> 2;                                 // its chunk
  const int sblk = u & 3;                               // its block inside the chunk
  const int n_diag = sblk + 1;                          // key blocks of the diagonal chunk
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + 16384;                              // [2][K 16 KB | V 16 KB] -> 2 x 32 KB
  uint8_t* sSnap = sKV + 2 * 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSnap + kAppSnapStages * kAppSnapBytes);
  uint64_t* q_full = bars;
  uint64_t* sn_full = q_full + 1;
  uint64_t* sn_empty = sn_full + kAppSnapStages;
  uint64_t* phi_full = sn_empty + kAppSnapStages;
  uint64_t* phi_empty = phi_full + kAppPhiBufs;
  uint64_t* kv_full = phi_empty + kAppPhiBufs;  // [2]
  uint64_t* kv_empty = kv_full + 2;             // [2]
  uint64_t* s_full = kv_empty + 2;
  uint64_t* p_full = s_full + 1;
  uint64_t* pv_done = p_full + 1;
  uint64_t* inter_done = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(inter_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kAppSnapStages; ++i) { mbar_init(sn_full + i, 1); mbar_init(sn_empty + i, 1); }
    for (int i = 0; i < kAppPhiBufs; ++i) { mbar_init(phi_full + i, 128); mbar_init(phi_empty + i, 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(kv_full + i, 1); mbar_init(kv_empty + i, 1); }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(inter_done, 2);  // both feature-block issuers
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: inter acc [0, 80) | diag acc [80, 160) | phi_q [160, 224) [224, 288) | S [288, 416) | P [416, 480)
  // The odd feature blocks accumulate in the diag columns first; the epilogue
  // warps move that partial to registers before they write the diagonal's P,
  // so the diagonal P.V (which needs P) cannot overwrite it early.
  const uint32_t t_inter = tmem, t_diag = tmem + 80, t_phi = tmem + 160, t_s = tmem + 288, t_p = tmem + 416;
  const int row0 = bh * p.S;
  const int snap_row0 = (bh * (n_chunks - p.prefix_chunks) + (c - p.prefix_chunks)) * kPolyN;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmSnap);
      mbar_expect_tx(q_full, 16384);
      tma_load_2d(sQ, &tmQ, q_full, 0, row0 + u * 128);
      for (int kb = 0; kb < kPolyFeatBlocks; ++kb) {
        const int st = kb % kAppSnapStages;
        if (!mbar_wait(sn_empty + st, ((kb / kAppSnapStages) & 1) ^ 1, p.err, kErrPolyWait)) return;
        mbar_expect_tx(sn_full + st, kAppSnapBytes);
        tma_load_2d(sSnap + st * kAppSnapBytes, &tmSnap, sn_full + st, kb * 128, snap_row0);
        tma_load_2d(sSnap + st * kAppSnapBytes + 10240, &tmSnap, sn_full + st, kb * 128 + 64, snap_row0);
      }
      for (int j = 0; j < n_diag; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty + st, ((j >> 1) & 1) ^ 1, p.err, kErrPolyWait)) return;
        mbar_expect_tx(kv_full + st, 32768);
        tma_load_2d(sKV + st * 32768, &tmK, kv_full + st, 0, row0 + (c * 4 + j) * 128);
        tma_load_2d(sKV + st * 32768 + 16384, &tmV, kv_full + st, 0, row0 + (c * 4 + j) * 128);
      }
    }
  } else if (warp == 1 || warp == 2) {
    {  // the whole warp: every wait agrees in all lanes; tcgen05 issues come from the elected lane
      constexpr uint32_t idesc_inter = idesc_f16_f32(128, kPolyN, false, false);
      constexpr uint32_t idesc_s = idesc_f16_f32(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, 64, false, true);
      bool ok = true;
      // phase 1: inter = phi_q(q) @ S_c over 33 feature blocks; phi_q is the
      // TMEM A operand (TS form), so only the snapshot passes through smem.
      // Warp 1 takes the even blocks (phi buffer 0) into the inter columns,
      // warp 2 the odd ones (buffer 1) into the diag columns.
      const int first_kb = warp - 1;
      const uint32_t t_acc = warp == 1 ? t_inter : t_diag;
      for (int kb = first_kb; kb < kPolyFeatBlocks && ok; kb += 2) {
        const int st = kb % kAppSnapStages, pb = kb % kAppPhiBufs;
        if (!mbar_wait_warp(sn_full + st, (kb / kAppSnapStages) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        if (!mbar_wait_warp(phi_full + pb, (kb / kAppPhiBufs) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t phi = t_phi + pb * 64;
        const uint32_t sn = smem_u32(sSnap + st * kAppSnapBytes);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // K = 128 features, 16 per MMA (8 TMEM columns)
          const uint64_t bd = smem_desc(sn + (ks >> 2) * 10240 + (ks & 3) * 32, 16, 1024, 128);
          umma_f16_ts_elect(t_acc, phi + ks * 8, bd, idesc_inter, (kb != first_kb || ks != 0));
        }
        umma_commit_elect(sn_empty + st);
        umma_commit_elect(phi_empty + pb);
      }
      if (ok) umma_commit_elect(inter_done);
      // phase 2 (warp 1): diagonal block, exact exp
      if (warp != 1) ok = false;
      if (ok && !mbar_wait_warp(q_full, 0, p.err, kErrPolyWait)) ok = false;
      const uint32_t qa = smem_u32(sQ);
      for (int j = 0; j < n_diag && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait_warp(kv_full + st, (j >> 1) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        if (j > 0 && !mbar_wait_warp(pv_done, (j - 1) & 1, p.err, kErrPolyWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + st * 32768);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = smem_desc(qa + ks * 32, 16, 1024, 128);
          const uint64_t bd = smem_desc(ka + ks * 32, 16, 1024, 128);
          umma_f16_ss_elect(t_s, ad, bd, idesc_s, ks != 0);
        }
        umma_commit_elect(s_full);
        if (!mbar_wait_warp(p_full, j & 1, p.err, kErrPolyWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t va = ka + 16384;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t bv = smem_desc(va + ks * 2048, 8192, 1024, 128);
          umma_f16_ts_elect(t_diag, t_p + ks * 8, bv, idesc_pv, (j | ks) != 0);
        }
        umma_commit_elect(pv_done);
        umma_commit_elect(kv_empty + st);
      }
    }
  } else {
    // ---------------------------------------------------- phi_q producer, diag exp, epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row (TMEM lane) of this thread
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    PolyCtl ctl = *p.ctl;
    const float rs = sqrtf(p.scale);
    bool ok = mbar_wait(q_full, 0, p.err, kErrPolyWait);
    uint32_t hrow[32];
    if (ok) load_row_h2(sQ, r, hrow);
    for (int kb = 0; kb < kPolyFeatBlocks && ok; ++kb) {
      const int pb = kb % kAppPhiBufs;
      if (!mbar_wait(phi_empty + pb, ((kb / kAppPhiBufs) & 1) ^ 1, p.err, kErrPolyWait)) { ok = false; break; }
      tc_fence_after();
      const float2 xi = kb < 32 ? load_pair(sQ, r, 2 * kb) : make_float2(0.f, 0.f);
      // this query row's 128 features as 64 fp16 pairs -> its TMEM lane
      uint32_t w[32];
      const float c_a = kb < 32 ? ctl.c2 * p.scale * xi.x : ctl.c1 * rs;
      scale_row_h2(hrow, c_a, w);
      tmem_st32(t_phi + pb * 64 + lane_off, w);
      if (kb < 32) {
        scale_row_h2(hrow, ctl.c2 * p.scale * xi.y, w);
      } else {
        const __half2 c0p = __floats2half2_rn(ctl.c0, 0.f);
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = 0u;
        w[0] = *reinterpret_cast<const uint32_t*>(&c0p);
      }
      tmem_st32(t_phi + pb * 64 + lane_off + 32, w);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(phi_full + pb);
    }
    // the odd feature blocks' partial (in the diag columns) -> registers
    uint32_t b0[32], b1[32];
    float den_b = 0.f;
    if (ok && mbar_wait(inter_done, 0, p.err, kErrPolyWait)) {
      tc_fence_after();
      uint32_t e[32];
      tmem_ld32(t_diag + lane_off, b0);
      tmem_ld32(t_diag + lane_off + 32, b1);
      tmem_ld32(t_diag + lane_off + 64, e);
      tmem_ld_wait();
      den_b = __uint_as_float(e[0]);
    } else {
      ok = false;
    }
    float diag_den = 0.f;  // this query's sum of exp over the diagonal block
    for (int j = 0; j < n_diag && ok; ++j) {
      if (!mbar_wait(s_full, j & 1, p.err, kErrPolyWait)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      tmem_ld32(t_s + lane_off + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
      tmem_ld32(t_s + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_ld32(t_s + lane_off + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
      tmem_ld32(t_s + lane_off + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
      tmem_ld_wait();
      const int lim = (j == sblk) ? r : 127;  // causal inside the chunk
      const float sl2 = p.scale * 1.4426950408889634f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float v0 = fminf(__uint_as_float(s[2 * i]) * sl2, kPolyMaxScore * 1.4426950408889634f);
        float v1 = fminf(__uint_as_float(s[2 * i + 1]) * sl2, kPolyMaxScore * 1.4426950408889634f);
        const float p0 = (2 * i <= lim) ? fast_exp2(v0) : 0.f;
        const float p1 = (2 * i + 1 <= lim) ? fast_exp2(v1) : 0.f;
        diag_den += p0 + p1;
        s[i] = pack_half2(p0, p1);
      }
      tmem_st32(t_p + lane_off, *reinterpret_cast<uint32_t(*)[32]>(s));
      tmem_st32(t_p + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
      // the next S overwrites the S columns only after PV(j) (waited by the MMA thread)
    }
    if (ok && (n_diag == 0 || mbar_wait(pv_done, (n_diag - 1) & 1, p.err, kErrPolyWait))) {
      tc_fence_after();
      const float t_prev = p.t_before + (float)(c * kPolyChunk);
      uint32_t a0[32], a1[32], d0[32], d1[32];
      tmem_ld32(t_inter + lane_off, a0);
      tmem_ld32(t_inter + lane_off + 32, a1);
      tmem_ld32(t_diag + lane_off, d0);
      tmem_ld32(t_diag + lane_off + 32, d1);
      tmem_ld_wait();
      uint32_t e[32];
      tmem_ld32(t_inter + lane_off + 64, e);
      tmem_ld_wait();
      const float den = t_prev * (__uint_as_float(e[0]) + den_b) + diag_den;
#pragma unroll
      for (int i = 0; i < 32; ++i) {  // even + odd feature-block partials
        a0[i] = __float_as_uint(__uint_as_float(a0[i]) + __uint_as_float(b0[i]));
        a1[i] = __float_as_uint(__uint_as_float(a1[i]) + __uint_as_float(b1[i]));
      }
      const float inv = 1.0f / den;
      const int qrow = u * 128 + r;
      __half* dst = p.ctx + ((size_t)b * p.S + qrow) * p.d_model + (size_t)h * 64;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 w;
        w.x = pack_half2((t_prev * __uint_as_float(a0[i]) + __uint_as_float(d0[i])) * inv,
                         (t_prev * __uint_as_float(a0[i + 1]) + __uint_as_float(d0[i + 1])) * inv);
        w.y = pack_half2((t_prev * __uint_as_float(a0[i + 2]) + __uint_as_float(d0[i + 2])) * inv,
                         (t_prev * __uint_as_float(a0[i + 3]) + __uint_as_float(d0[i + 3])) * inv);
        w.z = pack_half2((t_prev * __uint_as_float(a0[i + 4]) + __uint_as_float(d0[i + 4])) * inv,
                         (t_prev * __uint_as_float(a0[i + 5]) + __uint_as_float(d0[i + 5])) * inv);
        w.w = pack_half2((t_prev * __uint_as_float(a0[i + 6]) + __uint_as_float(d0[i + 6])) * inv,
                         (t_prev * __uint_as_float(a0[i + 7]) + __uint_as_float(d0[i + 7])) * inv);
        *reinterpret_cast<uint4*>(dst + i) = w;
        uint4 w2;
        w2.x = pack_half2((t_prev * __uint_as_float(a1[i]) + __uint_as_float(d1[i])) * inv,
                          (t_prev * __uint_as_float(a1[i + 1]) + __uint_as_float(d1[i + 1])) * inv);
        w2.y = pack_half2((t_prev * __uint_as_float(a1[i + 2]) + __uint_as_float(d1[i + 2])) * inv,
                          (t_prev * __uint_as_float(a1[i + 3]) + __uint_as_float(d1[i + 3])) * inv);
        w2.z = pack_half2((t_prev * __uint_as_float(a1[i + 4]) + __uint_as_float(d1[i + 4])) * inv,
                          (t_prev * __uint_as_float(a1[i + 5]) + __uint_as_float(d1[i + 5])) * inv);
        w2.w = pack_half2((t_prev * __uint_as_float(a1[i + 6]) + __uint_as_float(d1[i + 6])) * inv,
                          (t_prev * __uint_as_float(a1[i + 7]) + __uint_as_float(d1[i + 7])) * inv);
        *reinterpret_cast<uint4*>(dst + 32 + i) = w2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ shard fix-up
// Sequence sharding: fold the state of all earlier shards into this shard's
// snapshots.  gathered = every shard's total state [world][B*H][80][4224]
// fp32; local snapshot c holds the mean over this shard's first 512c tokens;
// afterwards it holds the mean over all tokens before its chunk.
// Heads bh0 .. bh0 + BH - 1; gathered = every shard's total of those heads,
// [world][BH][80][4224].
__global__ void __launch_bounds__(256) poly_fixup_kernel(const float* __restrict__ gathered, int rank, int BH,
                                                          int bh0, __half* __restrict__ snap, int n_snap,
                                                          int prefix_chunks, float t_before) {
  // Eight consecutive state elements per thread: the earlier shards' sum is
  // formed once (two float4 loads per shard), then every snapshot of those
  // elements is rewritten with one 16-byte load and store.  Memory-bound:
  // each rank reads and writes all of its snapshots once.
  const size_t per = (size_t)kPolyN * kPolyFeat;  // a multiple of 8
  const size_t total = (size_t)BH * per;
  const size_t per8 = per / 8;
  for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < total / 8; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    float before[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < rank; ++r) {
      const float4* g = reinterpret_cast<const float4*>(gathered + (size_t)r * total + e);
      const float4 a = __ldg(g), b = __ldg(g + 1);
      before[0] += a.x; before[1] += a.y; before[2] += a.z; before[3] += a.w;
      before[4] += b.x; before[5] += b.y; before[6] += b.z; before[7] += b.w;
    }
    const size_t bh = bh0 + e / per, rem = e - (e / per) * per;
    uint4* sp = reinterpret_cast<uint4*>(snap + bh * n_snap * per + rem);
#pragma unroll 4
    for (int i = 0; i < n_snap; ++i) {
      const float t_loc = (float)((prefix_chunks + i) * kPolyChunk);
      const float inv = 1.0f / (t_loc + t_before);
      uint4 w = sp[(size_t)i * per8];
      uint32_t* h = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[k]));
        const __half2 o = __floats2half2_rn((f.x * t_loc + before[2 * k]) * inv, (f.y * t_loc + before[2 * k + 1]) * inv);
        h[k] = *reinterpret_cast<const uint32_t*>(&o);
      }
      sp[(size_t)i * per8] = w;
    }
  }
}

}  // namespace tj
