// Persistent warp-specialised tcgen05 GEMM with fused epilogues.
//
//   C[M, N] = A[M, K] * W[N, K]^T     (A, W fp16 K-major; fp32 accumulate in TMEM)
//
// One CTA per SM.  Warp 0 issues TMA loads into a STAGES-deep shared-memory
// ring, warp 1 (its elected lane) issues tcgen05.mma into one of two TMEM
// accumulators, warps 2..9 drain the other accumulator through the epilogue
// (tcgen05.ld -> bias / GELU / residual / head scatter -> shared-memory
// transpose -> whole-line global stores).  Two epilogue warps share each TMEM
// lane quarter, one per half of the tile's columns; the residual epilogue
// prefetches the next 32-column chunk's residual while the current chunk is
// stored.  M tiles that hold no valid token (right
// padding) are dropped up front: the kernel walks a compact device-side list
// of live 128-row tiles.
#pragma once
#include "tj_common.cuh"

namespace tj {

enum EpiKind : int { kEpiQKV = 0, kEpiGelu = 1, kEpiResid = 2, kEpiPlain16 = 3 };

struct GemmParams {
  int M, N, K;
  int seq;               // rows per sample (row -> (b, n) = (row / seq, row % seq))
  const int* lengths;    // [B] valid-prefix length per sample
  const uint8_t* mask;   // [B*seq] per-row validity, or null (prefix lengths only)
  const int* tile_list;  // live 128-row tile indices
  const int* n_live;     // number of entries in tile_list
  const float* bias;     // [N]
  // kEpiQKV: Q,K,V as [B, H, seq, hd] fp16
  __half* q;
  __half* k;
  __half* v;
  int heads, head_dim, d_model;
  // kEpiGelu / kEpiPlain16: out16 [M, N]
  __half* out16;
  // kEpiResid: out32[row, :] = resid[row, :] + acc + bias (resid may alias out32)
  float* out32;
  const float* resid;
  int* err;
  // Packed rows (varlen): GEMM row r is the r-th valid token, at padded row
  // row_of[r] of the [B*seq] layout (-1 past the last valid token).  The
  // fp16 operand / output rows are packed; the QKV scatter and the FP32
  // residual stream go through row_of.  Null: rows are the padded rows.
  const int* row_of;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of fp16

// Epilogue staging: per epilogue warp 16 rows x 36 floats (FP32 residual
// epilogue: 32 + 4 padding, so both the row-per-lane writes and the
// column-per-lane reads of 16-byte words are bank-conflict free; the fp16
// epilogues use 16 rows x 80 bytes of it).
constexpr int kEpiStageFloats = 16 * 36;
constexpr int kEpiStageBytes = 8 * kEpiStageFloats * 4;

template <int BN>
struct GemmCfg {
  static constexpr int kStageA = kGemmBM * kGemmBK * 2;
  static constexpr int kStageB = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (200 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ + kEpiStageBytes;
  static constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps
  static constexpr int kEpiThreads = 256;
};

// Padded row of GEMM row `row`, or -1 for a row that holds no valid token.
TJ_DEV int src_row(const GemmParams& p, int row) {
  if (row >= p.M) return -1;
  if (p.row_of != nullptr) return p.row_of[row];
  const int b = row / p.seq;
  const int n = row - b * p.seq;
  if (n >= p.lengths[b]) return -1;
  return (p.mask == nullptr || __ldg(p.mask + row) != 0) ? row : -1;
}

TJ_DEV bool row_is_valid(const GemmParams& p, int row) {
  if (row >= p.M) return false;
  if (p.row_of != nullptr) return p.row_of[row] >= 0;
  const int b = row / p.seq;
  const int n = row - b * p.seq;
  if (n >= p.lengths[b]) return false;
  return p.mask == nullptr || __ldg(p.mask + row) != 0;
}

// Exact-form GELU 0.5 x (1 + erf(x / sqrt 2)) with erf from Abramowitz &
// Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7.
// Two SFU ops (reciprocal, exp2) and ~12 FMAs, no branches; for x < 0 the
// 1 + erf term is the series itself (no cancellation).  The resulting GELU is
// within 5e-7 of the exact one, far below the fp16 rounding of the output.
// Evaluated for two values at once on packed two-lane FP32 instructions
// (each lane rounds like the scalar operation; half the FMA/MUL issue slots).
TJ_DEV float2 gelu_erf_x2(float x0, float x1) {
  const uint64_t z = fmul_x2(f32x2(fabsf(x0), fabsf(x1)), f32x2(0.70710678118654752440f, 0.70710678118654752440f));
  const float2 den = f32x2_split(ffma_x2(f32x2(0.3275911f, 0.3275911f), z, f32x2(1.0f, 1.0f)));
  float t0, t1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(den.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(den.y));
  const uint64_t t = f32x2(t0, t1);
  uint64_t q = ffma_x2(t, f32x2(1.061405429f, 1.061405429f), f32x2(-1.453152027f, -1.453152027f));
  q = ffma_x2(t, q, f32x2(1.421413741f, 1.421413741f));
  q = ffma_x2(t, q, f32x2(-0.284496736f, -0.284496736f));
  q = ffma_x2(t, q, f32x2(0.254829592f, 0.254829592f));
  const uint64_t poly = fmul_x2(t, q);
  const float2 arg = f32x2_split(fmul_x2(fmul_x2(z, z), f32x2(-1.4426950408889634f, -1.4426950408889634f)));
  const float2 pe = f32x2_split(fmul_x2(poly, f32x2(fast_exp2(arg.x), fast_exp2(arg.y))));
  return make_float2(0.5f * x0 * (x0 >= 0.0f ? 2.0f - pe.x : pe.x), 0.5f * x1 * (x1 >= 0.0f ? 2.0f - pe.y : pe.y));
}

// fp16 epilogue (bias, then GELU or nothing; QKV scatter or row-major
// store) of one epilogue warp's 32 rows x kChunks 32-column chunks.  Each
// chunk's packed 64-byte row pieces go through shared memory (two rounds of
// 16 rows, 80-byte row pitch) so that each global store instruction writes
// eight rows' 64-byte pieces whole (lane l: row 8i + l/4, bytes 16(l%4)..+15)
// instead of 16 bytes in each of 32 rows.  Rows outside a sample's valid
// length are written as zeros, rows >= M not at all.
template <int EPI, int kChunks, typename WaitAcc>
TJ_DEV bool f16_epilogue(const GemmParams& p, uint32_t taddr, int row0, int colh, bool live, float* stage_f,
                         int lane, WaitAcc&& wait_acc) {
  uint8_t* stage = reinterpret_cast<uint8_t*>(stage_f);
  const bool my_valid = live && row_is_valid(p, row0 + lane);  // this thread's accumulator row
  const int piece = lane & 3;
  uint32_t in_m = 0;  // bit 2h+i: store-side row row0 + 16h + 8i + lane/4 is < M
  // QKV: element offset of that row's token (b, n) in head 0 of Q/K/V
  // [B, H, seq, hd], or -1 (a packed row past the last valid token); worked
  // out under the main loop so the stores need no division
  long long tok_ofs[4];
  if (live) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int row = row0 + 8 * k + (lane >> 2);
      tok_ofs[k] = -1;
      if (row < p.M) {
        in_m |= 1u << k;
        if constexpr (EPI == kEpiQKV) {
          const int pr = p.row_of != nullptr ? p.row_of[row] : row;
          if (pr >= 0) {
            const int b = pr / p.seq;
            tok_ofs[k] = ((long long)b * p.heads * p.seq + (pr - b * p.seq)) * p.head_dim;
          }
        }
      }
    }
  }
  // the bias of the next chunk is loaded one chunk ahead (chunk 0's under
  // the accumulator wait), so its latency hides behind the current chunk
  float4 bias_next[8];
  auto load_bias = [&](int c) {
    if (colh + c * 32 >= p.N) return;
#pragma unroll
    for (int j = 0; j < 8; ++j) bias_next[j] = __ldg(reinterpret_cast<const float4*>(p.bias + colh + c * 32) + j);
  };
  if (live) load_bias(0);
  if (!wait_acc()) return false;
  tc_fence_after();
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    float4 bias_cur[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) bias_cur[j] = bias_next[j];
    if (live && c + 1 < kChunks) load_bias(c + 1);
    uint32_t acc[32];
    tmem_ld32(taddr + c * 32, acc);
    tmem_ld_wait();
    const int col0 = colh + c * 32;
    if (!live || col0 >= p.N) continue;  // warp-uniform
    uint32_t w[16];
    if (my_valid) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 bb = bias_cur[j];
        float v0 = __uint_as_float(acc[4 * j]) + bb.x, v1 = __uint_as_float(acc[4 * j + 1]) + bb.y;
        float v2 = __uint_as_float(acc[4 * j + 2]) + bb.z, v3 = __uint_as_float(acc[4 * j + 3]) + bb.w;
        if constexpr (EPI == kEpiGelu) {
          const float2 g01 = gelu_erf_x2(v0, v1), g23 = gelu_erf_x2(v2, v3);
          v0 = g01.x; v1 = g01.y; v2 = g23.x; v3 = g23.y;
        }
        w[2 * j] = pack_half2(v0, v1);
        w[2 * j + 1] = pack_half2(v2, v3);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = 0u;
    }
    // column part of the destination (a 32-column chunk never straddles a head)
    __half* col_base;
    int which = 0, head = 0, dim0 = 0;
    if constexpr (EPI == kEpiQKV) {
      which = col0 / p.d_model;
      const int hc = col0 - which * p.d_model;
      head = hc / p.head_dim;
      dim0 = hc - head * p.head_dim;
      col_base = (which == 0 ? p.q : (which == 1 ? p.k : p.v)) + (size_t)head * p.seq * p.head_dim + dim0;
    } else {
      col_base = p.out16 + col0;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if ((lane >> 4) == h) {
        uint4* dst = reinterpret_cast<uint4*>(stage + (lane - 16 * h) * 80);
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rr = 8 * i + (lane >> 2);
        if ((in_m >> (2 * h + i)) & 1u) {
          const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * 80 + 16 * piece);
          const int row = row0 + 16 * h + rr;
          __half* dst = nullptr;
          if constexpr (EPI == kEpiQKV) {
            // packed rows scatter to their token's padded position; a packed
            // row past the last valid token has none
            const long long ofs = tok_ofs[2 * h + i];
            if (ofs >= 0) dst = col_base + ofs;
          } else {
            dst = col_base + (size_t)row * p.N;
          }
          if (dst != nullptr) *reinterpret_cast<uint4*>(dst + 8 * piece) = val;
        }
      }
      __syncwarp();
    }
  }
  return true;
}

// FP32 residual epilogue of one epilogue warp: its 32 accumulator rows x
// kChunks 32-column chunks (TMEM lane = row, one row per thread).  Each chunk
// is turned to a column-per-lane layout through shared memory (two rounds of
// 16 rows), so every global load of the residual and store of the result
// moves whole 128-byte lines (lane l: row 4i + l/8, columns 4(l%8)..+3); the
// next chunk's residual is loaded while the current one is stored.  Rows
// outside a sample's valid length are written as zeros, rows >= M not at all.
template <int kChunks, typename WaitAcc>
TJ_DEV bool resid_epilogue(const GemmParams& p, uint32_t taddr, int row0, int colh, bool live, float* stage,
                           int lane, WaitAcc&& wait_acc) {
  const int sub = lane >> 3;
  const int c4 = 4 * (lane & 7);
  uint32_t in_m = 0, valid = 0;  // bit i: row row0 + 4i + sub is written / valid
  int prow[8];                    // its row of the FP32 residual stream
#pragma unroll
  for (int i = 0; i < 8; ++i) prow[i] = row0 + 4 * i + sub;
  if (live) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = row0 + 4 * i + sub;
      if (row < p.M) {
        const int sr = src_row(p, row);
        if (p.row_of != nullptr) {
          prow[i] = sr;  // packed rows: only valid tokens have a residual row to write
          if (sr >= 0) in_m |= 1u << i;
        } else {
          in_m |= 1u << i;  // padded rows: invalid ones are written as zeros
        }
        if (sr >= 0) valid |= 1u << i;
      }
    }
  }
  // Pull this lane's row of the residual slice into L2 while the tile's MMAs
  // still run (one bulk prefetch, no registers); the register loads below
  // then wait on L2 rather than DRAM.  Only for short reductions (out-proj):
  // with K = 4096 the tile's own operand stream gains more from the L2.
  const int my_src = live && colh < p.N ? src_row(p, row0 + lane) : -1;
  if (p.K <= 1024 && my_src >= 0) {
    const float* src = p.resid + (size_t)my_src * p.N + colh;
    const int bytes = min(kChunks * 32, p.N - colh) * 4;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
  }
  float4 res[2][8];
  float4 bias4[2];  // this lane's 4 bias columns of the chunk, loaded with its residual
  auto prefetch = [&](int c, float4 (&r)[8]) {
    const int col = colh + c * 32 + c4;
    if (colh + c * 32 >= p.N) return;
    bias4[c & 1] = __ldg(reinterpret_cast<const float4*>(p.bias + col));
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((valid >> i) & 1u) r[i] = *reinterpret_cast<const float4*>(p.resid + (size_t)prow[i] * p.N + col);
  };
  if (live) prefetch(0, res[0]);  // overlaps the tile's last MMAs
  if (!wait_acc()) return false;
  tc_fence_after();
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    if (live && c + 1 < kChunks) prefetch(c + 1, res[(c + 1) & 1]);
    uint32_t acc[32];
    tmem_ld32(taddr + c * 32, acc);
    tmem_ld_wait();
    const int col0 = colh + c * 32;
    if (!live || col0 >= p.N) continue;  // warp-uniform
    const float4 b4 = bias4[c & 1];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if ((lane >> 4) == h) {
        float* dst = stage + (lane - 16 * h) * 36;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(dst + 4 * k) =
              make_float4(__uint_as_float(acc[4 * k]), __uint_as_float(acc[4 * k + 1]),
                          __uint_as_float(acc[4 * k + 2]), __uint_as_float(acc[4 * k + 3]));
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ii = 4 * h + i;
        const int rr = 4 * i + sub;
        if ((in_m >> ii) & 1u) {
          const float4 a = *reinterpret_cast<const float4*>(stage + rr * 36 + c4);
          float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
          if ((valid >> ii) & 1u) {
            const float4 r = res[c & 1][ii];
            o = make_float4(a.x + b4.x + r.x, a.y + b4.y + r.y, a.z + b4.z + r.z, a.w + b4.w + r.w);
          }
          *reinterpret_cast<float4*>(p.out32 + (size_t)prow[ii] * p.N + col0 + c4) = o;
        }
      }
      __syncwarp();
    }
  }
  return true;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full = bars;             // [S]
  uint64_t* empty = bars + S;        // [S]
  uint64_t* acc_full = bars + 2 * S; // [2]
  uint64_t* acc_empty = acc_full + 2;// [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* stage = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256) +
                 (threadIdx.x / 32 - 2) * kEpiStageFloats;  // epilogue warps 2..9

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(acc_full + i, 1); mbar_init(acc_empty + i, Cfg::kEpiThreads); }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // operands, tile list and residual come from earlier kernels

  const int n_tiles = (p.N + BN - 1) / BN;
  const int total = *p.n_live * n_tiles;
  const int k_blocks = (p.K + kGemmBK - 1) / kGemmBK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int mt = p.tile_list[t / n_tiles];
      const int nt = t % n_tiles;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait(empty + stage, phase ^ 1u, p.err, kErrGemmProducer)) { ok = false; break; }
        uint8_t* sa = smem + stage * Cfg::kStageBytes;
        uint8_t* sb = sa + Cfg::kStageA;
        mbar_expect_tx(full + stage, Cfg::kStageBytes);
        tma_load_2d(sa, &tmA, full + stage, kb * kGemmBK, mt * kGemmBM);
        tma_load_2d(sb, &tmW, full + stage, kb * kGemmBK, nt * BN);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
    // every load of this CTA is issued: the next kernel may launch and run
    // its prologue while the last tiles drain
    griddep_launch_dependents();
  } else if (warp == 1) {  // whole warp; tcgen05 issues from the elected lane
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(kGemmBM, BN, false, false);
    int stage = 0;
    uint32_t phase = 0;
    int abuf = 0;
    uint32_t aphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      if (!mbar_wait_warp(acc_empty + abuf, aphase ^ 1u, p.err, kErrGemmMma)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + abuf * BN;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait_warp(full + stage, phase, p.err, kErrGemmMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
        const uint32_t sb = sa + Cfg::kStageA;
#pragma unroll
        for (int ks = 0; ks < kGemmBK / 16; ++ks) {
          const uint64_t ad = smem_desc(sa + ks * 32, 16, 1024, 128);
          const uint64_t bd = smem_desc(sb + ks * 32, 16, 1024, 128);
          umma_f16_ss_elect(d_tmem, ad, bd, idesc, (kb | ks) != 0);
        }
        umma_commit_elect(empty + stage);  // release the smem stage when these MMAs retire
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      umma_commit_elect(acc_full + abuf);
      if (++abuf == 2) { abuf = 0; aphase ^= 1u; }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;     // which half of the tile's columns
    constexpr int kChunks = BN / 64;      // 32-column chunks per half
    int abuf = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int mt = p.tile_list[t / n_tiles];
      const int nt = t % n_tiles;
      const int row0 = mt * kGemmBM + quarter * 32;
      const int colh = nt * BN + half * (BN / 2);
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN + half * (BN / 2);
      auto wait_acc = [&] { return mbar_wait(acc_full + abuf, aphase, p.err, kErrGemmEpilogue); };
      bool ok;
      if constexpr (EPI == kEpiResid)
        ok = resid_epilogue<kChunks>(p, taddr, row0, colh, true, stage, lane, wait_acc);
      else
        ok = f16_epilogue<EPI, kChunks>(p, taddr, row0, colh, true, stage, lane, wait_acc);
      if (!ok) break;
      tc_fence_before();
      mbar_arrive(acc_empty + abuf);
      if (++abuf == 2) { abuf = 0; aphase ^= 1u; }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

// ------------------------------------------------------------------ 2-SM variant
// A cluster of 2 CTAs computes 256 x 256 output tiles with tcgen05.mma
// cta_group::2: each CTA stages its own 128 rows of A and 128 of the 256 W
// rows (32 KB per 64-deep k-block instead of 48 KB for a 128 x 256 tile),
// which buys a 6-deep ring in the same shared memory.  The pair may take any
// two live 128-row tiles (they need not be adjacent); an odd live count
// leaves the last pair's second half reading the zero-filled rows past M.
//   warp 0: TMA (both CTAs; completion on the even CTA's `full` barrier)
//   warp 1: the even CTA's warp issues the 2-SM MMAs from its elected lane;
//           commits are multicast to both CTAs (smem slot free / accumulator ready)
//   warps 2..9: epilogue of this CTA's 128 rows; done -> even CTA's acc_empty
struct Gemm2Cfg {
  static constexpr int kBN = 256;                       // N per pair tile (128 W rows per CTA)
  static constexpr int kStageBytes = 2 * kGemmBM * kGemmBK * 2;  // A 16 KB + W half 16 KB
  static constexpr int kStages = 6;
  static constexpr int kTmemCols = 512;                 // 2 x 256-column accumulators
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kEpiStageBytes;
  static constexpr int kThreads = 320;
  static constexpr int kEpiThreads = 256;
};

template <int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    const GemmParams p) {
  using Cfg = Gemm2Cfg;
  constexpr int S = Cfg::kStages;
  constexpr int BN = Cfg::kBN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full = bars;              // [S]  (even CTA's copy is the live one)
  uint64_t* empty = bars + S;         // [S]
  uint64_t* acc_full = bars + 2 * S;  // [2]
  uint64_t* acc_empty = acc_full + 2; // [2] (even CTA's copy is the live one)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* stage = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256) +
                 (threadIdx.x / 32 - 2) * kEpiStageFloats;  // epilogue warps 2..9

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0 = even CTA (issues the MMAs)
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(acc_full + i, 1); mbar_init(acc_empty + i, 2 * Cfg::kEpiThreads); }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive or multicast commit
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // operands, tile list and residual come from earlier kernels

  const int n_live = *p.n_live;
  const int n_tiles = p.N / BN;
  const int total = ((n_live + 1) >> 1) * n_tiles;  // pair tiles
  const int k_blocks = (p.K + kGemmBK - 1) / kGemmBK;
  // this CTA's 128-row tile of pair tile t (ghost tiles read rows past M: zero fill)
  auto my_mtile = [&](int t, bool& ghost) {
    const int li = 2 * (t / n_tiles) + (int)rank;
    ghost = li >= n_live;
    return ghost ? (p.M + kGemmBM - 1) / kGemmBM : p.tile_list[li];
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += n_pairs) {
      bool ghost;
      const int mt = my_mtile(t, ghost);
      const int nt = t % n_tiles;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait(empty + stage, phase ^ 1u, p.err, kErrGemmProducer)) { ok = false; break; }
        uint8_t* sa = smem + stage * Cfg::kStageBytes;
        uint8_t* sb = sa + kGemmBM * kGemmBK * 2;
        const uint32_t lb = pair_leader_bar(full + stage);
        if (rank == 0) mbar_expect_tx(full + stage, 2 * Cfg::kStageBytes);  // both CTAs' bytes
        tma_load_2d_pair(sa, &tmA, lb, kb * kGemmBK, mt * kGemmBM);
        tma_load_2d_pair(sb, &tmW, lb, kb * kGemmBK, nt * BN + (int)rank * 128);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
    griddep_launch_dependents();  // every load of this CTA is issued
  } else if (warp == 1 && rank == 0) {  // whole warp; tcgen05 issues from the elected lane
    // ------------------------------------------------------------ 2-SM MMA issuer (even CTA)
    constexpr uint32_t idesc = idesc_f16_f32(256, BN, false, false);
    int stage = 0;
    uint32_t phase = 0;
    int abuf = 0;
    uint32_t aphase = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += n_pairs) {
      if (!mbar_wait_warp(acc_empty + abuf, aphase ^ 1u, p.err, kErrGemmMma)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + abuf * BN;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait_warp(full + stage, phase, p.err, kErrGemmMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
        const uint32_t sb = sa + kGemmBM * kGemmBK * 2;
#pragma unroll
        for (int ks = 0; ks < kGemmBK / 16; ++ks) {
          const uint64_t ad = smem_desc(sa + ks * 32, 16, 1024, 128);
          const uint64_t bd = smem_desc(sb + ks * 32, 16, 1024, 128);
          umma_f16_ss_pair_elect(d_tmem, ad, bd, idesc, (kb | ks) != 0);
        }
        umma_commit_pair_both_elect(empty + stage);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      umma_commit_pair_both_elect(acc_full + abuf);
      if (++abuf == 2) { abuf = 0; aphase ^= 1u; }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int kChunks = BN / 64;
    const uint32_t leader_acc_empty0 = map_to_rank(acc_empty, 0);
    int abuf = 0;
    uint32_t aphase = 0;
    for (int t = pair; t < total; t += n_pairs) {
      bool ghost;
      const int mt = my_mtile(t, ghost);
      const int nt = t % n_tiles;
      const int row0 = mt * kGemmBM + quarter * 32;
      const int colh = nt * BN + half * (BN / 2);
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN + half * (BN / 2);
      auto wait_acc = [&] { return mbar_wait(acc_full + abuf, aphase, p.err, kErrGemmEpilogue); };
      bool ok;
      if constexpr (EPI == kEpiResid)
        ok = resid_epilogue<kChunks>(p, taddr, row0, colh, !ghost, stage, lane, wait_acc);
      else
        ok = f16_epilogue<EPI, kChunks>(p, taddr, row0, colh, !ghost, stage, lane, wait_acc);
      if (!ok) break;
      tc_fence_before();
      mbar_arrive_cluster(leader_acc_empty0 + (uint32_t)(abuf * sizeof(uint64_t)));
      if (++abuf == 2) { abuf = 0; aphase ^= 1u; }
    }
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair partner may still touch its barriers or smem
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

}  // namespace tj
