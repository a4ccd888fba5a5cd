// Flash-style causal / padded self-attention on tcgen05 with S, P and O in TMEM.
//
// One CTA per (pair of 128-query tiles, head, sample).  Q, K, V are fp16
// [B, H, S, HD] (written by the packed-QKV GEMM epilogue); the context is
// written fp16 into [B*S, d_model] at column h*HD so the output projection
// reads it directly.
//
//   warp 8       TMA producer: both Q tiles once, then K/V tiles into a ring
//   warps 9, 10  MMA issue (the elected lane of each converged warp), per
//                key tile j, for query tile t = warp - 9 (head_dim <= 64;
//                warp 9 issues both tiles for head_dim 128):
//                  S_t = Q_t K_j^T          (SS form, fp32 in TMEM)
//                  O_t += P_t V_j           (TS form: P_t read from TMEM)
//   warps 0..3   softmax for query tile 0, warps 4..7 for tile 1: thread r
//                owns row r; one pass over its S row (fp32, exp2 domain),
//                writes P (fp16, packed 2 per column) to TMEM (own columns
//                for head_dim <= 64, so S_t(j+1) overlaps this tile's
//                exponentials; over S for head_dim 128),
//                and rescales its O row in TMEM only when its running max
//                grows by more than 2^8 (stale maxima keep p <= 256).
//
// The two query tiles ping-pong: while one warpgroup exponentiates, the
// tensor core works on the other tile.  Key tiles above the causal diagonal
// are never visited; query tiles past a sample's valid length are skipped;
// with causal + right padding the key mask is provably redundant (every key
// <= a valid query is valid) and is not evaluated.  Rows whose keys are all
// masked produce 0.
#pragma once
#include "tj_common.cuh"

namespace tj {

struct AttnParams {
  const int* lengths;      // [B]
  const uint8_t* mask;     // [B*S] key/row validity; used only for samples flagged general
  const uint8_t* general;  // [B] 1 if the sample's mask is not a right-padded prefix
  __half* ctx;             // [B*S, d_model]
  int S, H, d_model;
  int causal;
  float scale_log2;        // head_dim^-0.5 * log2(e)
  int* err;
  // Polynomial route: when *poly_admit != 0 only query pairs < exact_pairs
  // (the exact prefix) are computed here; null = every query.
  const int* poly_admit;
  int exact_pairs;
  // Sequence sharding: local query row 0 sits at global position q_pos0 and
  // K/V hold kv_shard rows per (shard, b, h): the key at global position pos
  // is row ((pos / kv_shard * B + b) * H + h) * kv_shard + pos % kv_shard.
  // Unsharded: q_pos0 = 0, kv_shard = S.
  // Zig-zag sharding (zz_chunk > 0, a multiple of 256): the sequence is cut
  // into 2 * kv_shards chunks of zz_chunk tokens and shard r holds chunks r
  // and 2 * kv_shards - 1 - r back to back (kv_shard = 2 * zz_chunk), so
  // every shard gets the same causal work; local query row zz_chunk sits at
  // global position q_pos1.
  int q_pos0;
  int kv_shard;
  int kv_shards;  // shards present in K/V (1 unless sharded)
  int zz_chunk;
  int q_pos1;
  int B;
  // Persistent kernel's work scheduler: {next item, CTAs finished}, zero
  // before the launch and zero again after it (the last CTA to finish resets
  // both).  Null: item i goes to CTA i % grid.
  int* sched;
  // Varlen packing: the context row of token (b, n) is pack_of[b*S + n]
  // (-1: padding, not written).  Null: row b*S + n.
  const int* pack_of;
};

// Global 128-token tile of local query tile q (a tile never straddles a
// zig-zag chunk: zz_chunk is a multiple of 256, so neither does a pair).
TJ_DEV int q_global_tile(const AttnParams& p, int q) {
  const int r = q * 128;
  if (p.zz_chunk == 0 || r < p.zz_chunk) return (p.q_pos0 + r) / 128;
  return (p.q_pos1 + r - p.zz_chunk) / 128;
}
// First K/V row of the 128-key tile that starts at global position pos.
TJ_DEV int kv_tile_row(const AttnParams& p, int b, int h, int pos) {
  int shard, off;
  if (p.zz_chunk > 0) {
    const int c = pos / p.zz_chunk;
    const bool first = c < p.kv_shards;
    shard = first ? c : 2 * p.kv_shards - 1 - c;
    off = (first ? 0 : p.zz_chunk) + (pos - c * p.zz_chunk);
  } else {
    shard = pos / p.kv_shard;
    off = pos - shard * p.kv_shard;
  }
  return ((shard * p.B + b) * p.H + h) * p.kv_shard + off;
}

// Context row of query token (b, qrow), or -1 when it is not written.
TJ_DEV long long ctx_row(const AttnParams& p, int b, int qrow) {
  if (qrow >= p.S) return -1;
  const long long r = (long long)b * p.S + qrow;
  return p.pack_of != nullptr ? (long long)p.pack_of[r] : r;
}

template <int HD>
struct AttnCfg {
  static_assert(HD == 32 || HD == 64 || HD == 128, "head_dim must be 32, 64 or 128");
  static constexpr int kSw = HD >= 64 ? 128 : 64;  // swizzle span (bytes) of Q/K/V rows
  static constexpr int kRowB = kSw;                 // bytes per smem row inside one atom
  static constexpr int kAtomCols = kSw / 2;         // fp16 columns per atom
  static constexpr int kAtoms = HD / kAtomCols;
  static constexpr int kAtomBytes = 128 * kRowB;
  static constexpr int kTile = 128 * HD * 2;
  static constexpr int kStages = HD >= 128 ? 2 : (HD == 64 ? 4 : 6);
  static constexpr int kSmemBytes = 2 * kTile + kStages * 2 * kTile + 1024 + 256;
  static constexpr int kTmemCols = 512;
  // TMEM columns.  HD <= 64: S0 S1 (fp32) | P0 P1 (fp16 pairs) | O0 O1, so the
  // next S can be computed while P is still being consumed.  HD = 128: P
  // overwrites the first half of S (S0 S1 | O0 O1 fills all 512 columns).
  static constexpr bool kPSeparate = HD <= 64;
  static constexpr int kColS = 0;
  static constexpr int kColP = kPSeparate ? 256 : 0;
  static constexpr int kColO = kPSeparate ? 384 : 256;
  // TMA warp 8, MMA warp 9, 8 softmax warps; with P in its own columns a
  // second MMA warp (10) issues tile 1's S and PV.
  static constexpr int kThreads = HD <= 64 ? 352 : 320;
  static constexpr float kRescaleLog2 = 8.0f;
};

// Score-row masking (one thread = one query row of 128 key columns).
// Columns past `lim` (future keys on the diagonal tile, keys past the valid
// length on the tail tile) become -inf: a compare-and-select per column with
// no other live state, so the 128 scores stay in registers.
TJ_DEV void mask_past(uint32_t (&s)[128], int lim) {
#pragma unroll
  for (int i = 0; i < 128; ++i) s[i] = i > lim ? 0xff800000u : s[i];
}
// Columns whose key is masked out (general, non-prefix masks only).
TJ_DEV void mask_keys(uint32_t (&s)[128], const uint8_t* __restrict__ key_valid) {
#pragma unroll
  for (int i = 0; i < 128; ++i) s[i] = __ldg(key_valid + i) == 0 ? 0xff800000u : s[i];
}

template <int HD>
__global__ void __launch_bounds__(AttnCfg<HD>::kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<HD>;
  constexpr int ST = Cfg::kStages;
  griddep_launch_dependents();
  griddep_wait();  // Q/K/V and lengths come from earlier kernels
  const int bh = blockIdx.y;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int n_pairs = gridDim.x;
  const int pair = p.causal ? (n_pairs - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int len = p.lengths[b];  // valid keys (global positions)
  const int q0 = 2 * pair;               // local query tile of warpgroup 0
  const int qg0 = q_global_tile(p, q0);  // its global tile
  if (qg0 * 128 >= len || q0 * 128 >= p.S) return;
  if (error_raised(p.err)) return;
  if (p.poly_admit != nullptr && pair >= p.exact_pairs && *reinterpret_cast<const volatile int*>(p.poly_admit) != 0)
    return;
  const bool has1 = (qg0 + 1) * 128 < len && (q0 + 1) * 128 < p.S;
  const int kv_all = (len + 127) / 128;
  const int nkv0 = p.causal ? qg0 + 1 : kv_all;
  const int nkv1 = has1 ? (p.causal ? qg0 + 2 : kv_all) : 0;
  const int n_kv = nkv0 > nkv1 ? nkv0 : nkv1;
  const bool general = p.mask != nullptr && p.general[b] != 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [2][tile]
  uint8_t* sKV = sQ + 2 * Cfg::kTile;      // stage s: K at s*2*kTile, V after it
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + ST * 2 * Cfg::kTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;  // [2]
  uint64_t* p_full = s_full + 2;     // [2]
  uint64_t* pv_done = p_full + 2;    // [2]
  uint64_t* o_final = pv_done + 2;   // [2]
  uint64_t* s_free = o_final + 2;    // [2] softmax has read S_t into registers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ST; ++i) { mbar_init(kv_full + i, 1); mbar_init(kv_empty + i, Cfg::kPSeparate ? 2 : 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 128);
      mbar_init(pv_done + i, 1);
      mbar_init(o_final + i, 1);
      mbar_init(s_free + i, 128);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int row0 = bh * p.S;  // first Q row of this (b, h) in the [B*H*S, HD] view
  auto kv_row = [&](int j) { return kv_tile_row(p, b, h, j * 128); };  // key tile j (global positions j*128 ..)

  if (warp == 8) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_expect_tx(q_full, (has1 ? 2 : 1) * Cfg::kTile);
      for (int t = 0; t < (has1 ? 2 : 1); ++t)
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_2d(sQ + t * Cfg::kTile + a * Cfg::kAtomBytes, &tmQ, q_full, a * Cfg::kAtomCols,
                      row0 + (q0 + t) * 128);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(kv_empty + st, ((j / ST) & 1) ^ 1, p.err, kErrAttnProducer)) break;
        uint8_t* sk = sKV + st * 2 * Cfg::kTile;
        uint8_t* sv = sk + Cfg::kTile;
        mbar_expect_tx(kv_full + st, 2 * Cfg::kTile);
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a) {
          tma_load_2d(sk + a * Cfg::kAtomBytes, &tmK, kv_full + st, a * Cfg::kAtomCols, kv_row(j));
          tma_load_2d(sv + a * Cfg::kAtomBytes, &tmV, kv_full + st, a * Cfg::kAtomCols, kv_row(j));
        }
      }
    }
  } else if (warp == 9 || (Cfg::kPSeparate && warp == 10)) {
    {  // the whole warp: every wait agrees in all lanes; tcgen05 issues come from the elected lane
      // ---------------------------------------------------------- MMA issuer(s)
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait_warp(q_full, 0, p.err, kErrAttnMma);
      auto issue_s = [&](int t, int jj, uint32_t k_addr) {
        const uint32_t qa = q_addr + t * Cfg::kTile;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const int atom = (ks * 16) / Cfg::kAtomCols;
          const int within = ((ks * 16) % Cfg::kAtomCols) * 2;
          const uint64_t ad = smem_desc(qa + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
          const uint64_t bd = smem_desc(k_addr + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
          umma_f16_ss_elect(tmem + Cfg::kColS + t * 128, ad, bd, idesc_qk, ks != 0);
        }
        umma_commit_elect(s_full + t);
      };
      auto issue_pv = [&](int t, int jj, uint32_t v_addr) {
        const uint32_t o_tmem = tmem + Cfg::kColO + t * HD;
        const uint32_t p_tmem = tmem + (Cfg::kPSeparate ? Cfg::kColP + t * 64 : Cfg::kColS + t * 128);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t bd = smem_desc(v_addr + ks * 16 * Cfg::kRowB, Cfg::kAtomBytes, 8 * Cfg::kRowB, Cfg::kSw);
          umma_f16_ts_elect(o_tmem, p_tmem + ks * 8, bd, idesc_pv, (jj | ks) != 0);
        }
        umma_commit_elect(pv_done + t);
        if (jj == (t == 0 ? nkv0 : nkv1) - 1) umma_commit_elect(o_final + t);
      };
      auto kv_addr = [&](int jj) { return smem_u32(sKV + (jj % ST) * 2 * Cfg::kTile); };
      if constexpr (Cfg::kPSeparate) {
        // One issuing warp per query tile (warp 9: tile 0, warp 10: tile 1),
        // so neither tile's S or PV waits behind the other tile's softmax.
        // Per step j: S_t(j+1) as soon as the softmax has read S_t(j), then
        // PV_t(j) once P_t(j) is ready.  Both issuers release every K/V stage
        // (count 2): by a commit after their MMAs, or, for the steps past
        // their tile's last key tile, by a plain arrive once the stage landed.
        const int t = warp - 9;
        const int nkv_t = t == 0 ? nkv0 : nkv1;
        for (int j = 0; j < n_kv && ok; ++j) {
          const int st = j % ST;
          if (!mbar_wait_warp(kv_full + st, (j / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
          tc_fence_after();
          if (j >= nkv_t) {
            mbar_arrive_elect(kv_empty + st);
            continue;
          }
          if (j == 0) issue_s(t, 0, kv_addr(0));
          if (j + 1 < nkv_t) {
            const int sn = (j + 1) % ST;
            if (!mbar_wait_warp(kv_full + sn, ((j + 1) / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
            if (!mbar_wait_warp(s_free + t, j & 1, p.err, kErrAttnMma)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, j + 1, kv_addr(j + 1));
          }
          if (!mbar_wait_warp(p_full + t, j & 1, p.err, kErrAttnMma)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j, kv_addr(j) + Cfg::kTile);
          umma_commit_elect(kv_empty + st);
        }
      } else {
        // P_t(j) lives in S_t's columns: S_t(j+1) must wait for PV_t(j).
        for (int j = 0; j < n_kv && ok; ++j) {
          const int st = j % ST;
          if (!mbar_wait_warp(kv_full + st, (j / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
          tc_fence_after();
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= (t == 0 ? nkv0 : nkv1)) continue;
            if (j > 0 && !mbar_wait_warp(pv_done + t, (j - 1) & 1, p.err, kErrAttnMma)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, j, kv_addr(j));
          }
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= (t == 0 ? nkv0 : nkv1)) continue;
            if (!mbar_wait_warp(p_full + t, j & 1, p.err, kErrAttnMma)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, j, kv_addr(j) + Cfg::kTile);
          }
          umma_commit_elect(kv_empty + st);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;       // query tile of this warpgroup
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int nkv_t = t == 0 ? nkv0 : nkv1;
    const int r = quarter * 32 + lane;
    const int qt = q0 + t;
    const int qrow = qt * 128 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + Cfg::kColS + t * 128;
    const uint32_t p_col = tmem + lane_off + (Cfg::kPSeparate ? Cfg::kColP + t * 64 : Cfg::kColS + t * 128);
    const uint32_t o_col = tmem + lane_off + Cfg::kColO + t * HD;
    const float sl2 = p.scale_log2;
    const uint8_t* kmask = general ? p.mask + (size_t)b * p.S : nullptr;
    float m_run = -INFINITY;  // running (possibly stale) max, log2 units
    float l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv_t; ++j) {
      if (!mbar_wait(s_full + t, j & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      tmem_ld32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
      tmem_ld32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_ld32(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
      tmem_ld32(s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
      tmem_ld_wait();
      if constexpr (Cfg::kPSeparate) {
        tc_fence_before();
        mbar_arrive(s_free + t);  // S_t may now be overwritten by S_t(j+1)
      }
      const int kbase = j * 128;
      const bool diag = p.causal && j == qg0 + t;
      const bool tail = kbase + 128 > len;
      if (diag || tail) {
        const int lim_causal = diag ? r : 127;           // keys with col > lim are in the future
        const int lim_len = len - kbase - 1;             // keys with col > lim are past the length
        mask_past(s, lim_causal < lim_len ? lim_causal : lim_len);
      }
      if (general) mask_keys(s, kmask + kbase);
      const float mx = row_max128(s);
      const float m_tile = mx * sl2;
      const bool grow = m_tile > m_run + Cfg::kRescaleLog2;
      float alpha = 1.0f;
      if (grow) {
        alpha = fast_exp2(m_run - m_tile);  // 0 when m_run = -inf
        m_run = m_tile;
      }
      const float msub = m_run == -INFINITY ? 0.0f : m_run;
      // P packs two fp16 per 32-bit column, written over s[0..63]
      const float rowsum = exp_pack_rowsum(s, sl2, msub);
      if constexpr (Cfg::kPSeparate) {
        // P_t and O_t are free once PV_t(j-1) has retired
        if (j > 0 && !mbar_wait(pv_done + t, (j - 1) & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_st32(p_col, *reinterpret_cast<uint32_t(*)[32]>(s));
      tmem_st32(p_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      l_run = l_run * alpha + rowsum;
      // Rescale this row of O in TMEM (the whole warp takes part if any lane
      // needs it).  PV_t(j-1) has retired, so O is stable.
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_col + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full + t);
    }
    if (ok && nkv_t > 0 && mbar_wait(o_final + t, 0, p.err, kErrAttnSoftmax)) {
      tc_fence_after();
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      const long long crow = ctx_row(p, b, qrow);
      __half* dst = p.ctx + (crow < 0 ? 0 : crow) * (size_t)p.d_model + (size_t)h * HD;
      const bool store = crow >= 0;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_col + c * 32, o);
        tmem_ld_wait();
        if (store) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
            w.y = pack_half2(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            w.z = pack_half2(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            w.w = pack_half2(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + i) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace tj


namespace tj {

// ------------------------------------------------------------------ persistent warp-specialised kernel
// Same arithmetic per (pair of 128-query tiles, head, sample) work item as
// attn_fwd_kernel with head_dim <= 64 (P in its own TMEM columns), but one CTA
// per SM walks the items heavy-first: item i covers query-tile pair
// np-1 - i/BH of head-sample i%BH for causal attention.  With a scheduler
// (AttnParams::sched) CTAs claim items with an atomic counter, so each SM
// takes the next heaviest item when it frees up; without one CTA c takes
// items c, c + grid, ...  Roles (12 warps, three warpgroups):
//   warp 8       producer: claims the next live item, publishes it in a
//                4-slot ring, loads its two Q tiles (double-buffered across
//                items) and streams the K/V tiles through the stage ring
//   warp 9       issues S_t = Q_t K_j^T for both query tiles (SS form)
//   warps 10, 11 issue O_t += P_t V_j for query tile 0 / 1 (TS form)
//   warps 0..7   softmax, warpgroup t for query tile t (thread = query row)
// Three issuing warps keep the tensor pipe fed: a tcgen05.mma costs its
// issuing warp ~100 cycles whatever its size, so one warp issuing a tile's
// 4 + 8 MMAs per key tile serialises ~1.2k cycles of issue per step.  The
// softmax warpgroups get 224 registers per thread (the 128-column score row
// stays in registers, no spills) and the issuing warpgroup keeps 56:
// 2 x 224 + 56 = 3 x 168, the launch's register share.
// Item transitions overlap: the S issuer starts the next item's S_t(0) as
// soon as the softmax has read the last S_t, and the softmax warps
// exponentiate the next item's first key tile before they drain the previous
// item's O_t (normalise, store) -- the drain waits for that item's last P.V,
// which thereby runs under the exponentials.
template <int HD>
struct AttnPCfg {
  using Base = AttnCfg<HD>;
  static constexpr int kThreads = 384;
  static constexpr int kStages = HD == 64 ? 4 : 6;
  static constexpr int kItemSlots = 4;
  static constexpr int kRegLaunch = 168;  // 65536 / 384, rounded down to a multiple of 8
  static constexpr int kRegSoftmax = 224;
  static constexpr int kRegIssue = 56;
  static_assert(2 * kRegSoftmax + kRegIssue == 3 * kRegLaunch, "register split must use the launch's registers");
  static constexpr int kBarBytes = 8 * (14 + 2 * kStages + 2 * kItemSlots) + 4 * kItemSlots + 4;
  static_assert(kBarBytes <= 512, "barrier region");
  static constexpr int kSmemBytes = 4 * Base::kTile + kStages * 2 * Base::kTile + 1024 + 512;
};

template <int HD>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_persistent_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const AttnParams p, int n_pairs) {
  using Cfg = AttnCfg<HD>;
  using PC = AttnPCfg<HD>;
  static_assert(Cfg::kPSeparate, "persistent kernel needs P in its own TMEM columns");
  constexpr int ST = PC::kStages;
  constexpr int NI = PC::kItemSlots;
  const int BH = p.B * p.H;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [2 buffers][2 tiles][tile]
  uint8_t* sKV = sQ + 4 * Cfg::kTile;      // stage s: K at s*2*kTile, V after it
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + ST * 2 * Cfg::kTile);
  uint64_t* q_full = bars;                 // [2]
  uint64_t* q_empty = q_full + 2;          // [2]
  uint64_t* kv_full = q_empty + 2;         // [ST]
  uint64_t* kv_empty = kv_full + ST;       // [ST]
  uint64_t* s_full = kv_empty + ST;        // [2 tiles]
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* o_final = pv_done + 2;
  uint64_t* item_full = o_final + 2;       // [NI]
  uint64_t* item_empty = item_full + NI;   // [NI]
  int* item_slot = reinterpret_cast<int*>(item_empty + NI);  // [NI]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_slot + NI);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(q_full + i, 1); mbar_init(q_empty + i, 1); }
    // each K/V stage is released by the S issuer and both P.V issuers
    for (int i = 0; i < ST; ++i) { mbar_init(kv_full + i, 1); mbar_init(kv_empty + i, 3); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, 128);
      mbar_init(p_full + i, 128);
      mbar_init(pv_done + i, 1);
      mbar_init(o_final + i, 1);
    }
    // an item slot is read by the 11 consumer warps (8 softmax, 3 issuers)
    for (int i = 0; i < NI; ++i) { mbar_init(item_full + i, 1); mbar_init(item_empty + i, 11); }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // Q/K/V, lengths and the scheduler words come from earlier kernels
  const bool gated = p.poly_admit != nullptr && *reinterpret_cast<const volatile int*>(p.poly_admit) != 0;
  // an admitted polynomial route leaves only the exact prefix's pairs here
  const int np = gated ? min(n_pairs, p.exact_pairs) : n_pairs;
  const int n_items = np * BH;

  // Work item decode, identical in every role.
  struct Item {
    int b, h, bh, q0, qg0, len, nkv0, nkv1, n_kv;
    bool has1, general;
  };
  auto decode = [&](int i, Item& it) -> bool {
    const int pair = p.causal ? np - 1 - i / BH : i / BH;
    it.bh = i % BH;
    it.b = it.bh / p.H;
    it.h = it.bh - it.b * p.H;
    it.len = p.lengths[it.b];
    it.q0 = 2 * pair;
    it.qg0 = q_global_tile(p, it.q0);
    if (it.qg0 * 128 >= it.len || it.q0 * 128 >= p.S) return false;
    it.has1 = (it.qg0 + 1) * 128 < it.len && (it.q0 + 1) * 128 < p.S;
    const int kv_all = (it.len + 127) / 128;
    it.nkv0 = p.causal ? it.qg0 + 1 : kv_all;
    it.nkv1 = it.has1 ? (p.causal ? it.qg0 + 2 : kv_all) : 0;
    it.n_kv = it.nkv0 > it.nkv1 ? it.nkv0 : it.nkv1;
    it.general = p.mask != nullptr && p.general[it.b] != 0;
    return true;
  };
  auto kv_row = [&](const Item& it, int j) { return kv_tile_row(p, it.b, it.h, j * 128); };
  // Consumer side of the item ring (whole warp): the n-th published item, or
  // -1 once the producer has run out of work.
  auto next_item = [&](int n, int& item, int site) -> bool {
    const int slot = n % NI;
    if (!mbar_wait_warp(item_full + slot, (n / NI) & 1, p.err, site)) return false;
    int v = 0;
    if (lane == 0) v = *reinterpret_cast<volatile int*>(item_slot + slot);
    item = __shfl_sync(0xffffffffu, v, 0);
    mbar_arrive_elect(item_empty + slot);
    return true;
  };

  if (warp >= 8) {
    reg_dealloc<PC::kRegIssue>();
    if (warp == 8) {
      if (lane == 0) {
        // ---------------------------------------------------------- producer
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        int static_next = blockIdx.x;
        auto claim = [&]() {
          if (p.sched != nullptr) return atomicAdd(p.sched, 1);
          const int c = static_next;
          static_next += gridDim.x;
          return c;
        };
        // the next claim is issued as soon as the current item is known, so
        // its latency hides under this item's loads
        int pending = error_raised(p.err) ? n_items : claim();
        int kvc = 0;
        for (int n = 0;; ++n) {
          int item = -1;
          Item it;
          while (pending < n_items) {
            const int c = pending;
            pending = claim();
            if (decode(c, it)) { item = c; break; }
          }
          // nothing left to claim: this is the CTA's last item, so the next
          // kernel may launch and run its prologue while it finishes
          if (pending >= n_items) griddep_launch_dependents();
          const int slot = n % NI;
          if (n >= NI && !mbar_wait(item_empty + slot, ((n / NI) - 1) & 1, p.err, kErrAttnProducer)) break;
          item_slot[slot] = item;
          mbar_arrive(item_full + slot);
          if (item < 0) break;
          const int qb = n & 1;
          if (n >= 2 && !mbar_wait(q_empty + qb, ((n >> 1) - 1) & 1, p.err, kErrAttnProducer)) break;
          mbar_expect_tx(q_full + qb, (it.has1 ? 2 : 1) * Cfg::kTile);
          for (int t = 0; t < (it.has1 ? 2 : 1); ++t)
#pragma unroll
            for (int a = 0; a < Cfg::kAtoms; ++a)
              tma_load_2d(sQ + (qb * 2 + t) * Cfg::kTile + a * Cfg::kAtomBytes, &tmQ, q_full + qb,
                          a * Cfg::kAtomCols, it.bh * p.S + (it.q0 + t) * 128);
          bool ok = true;
          for (int j = 0; j < it.n_kv; ++j) {
            const int g = kvc + j, st = g % ST;
            if (!mbar_wait(kv_empty + st, ((g / ST) & 1) ^ 1, p.err, kErrAttnProducer)) { ok = false; break; }
            uint8_t* sk = sKV + st * 2 * Cfg::kTile;
            mbar_expect_tx(kv_full + st, 2 * Cfg::kTile);
#pragma unroll
            for (int a = 0; a < Cfg::kAtoms; ++a) {
              tma_load_2d(sk + a * Cfg::kAtomBytes, &tmK, kv_full + st, a * Cfg::kAtomCols, kv_row(it, j));
              tma_load_2d(sk + Cfg::kTile + a * Cfg::kAtomBytes, &tmV, kv_full + st, a * Cfg::kAtomCols,
                          kv_row(it, j));
            }
          }
          if (!ok) break;
          kvc += it.n_kv;
        }
      }
    } else if (warp == 9) {
      // ------------------------------------------------------------ S issuer (whole warp, elected lane issues)
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, 128, false, false);
      int kvc = 0;
      int cs[2] = {0, 0};  // S_t computed so far
      bool ok = true;
      for (int n = 0; ok; ++n) {
        int item;
        if (!next_item(n, item, kErrAttnMma) || item < 0) break;
        Item it;
        decode(item, it);
        const int qb = n & 1;
        if (!mbar_wait_warp(q_full + qb, (n >> 1) & 1, p.err, kErrAttnMma)) break;
        const uint32_t q_addr = smem_u32(sQ + qb * 2 * Cfg::kTile);
        for (int j = 0; j < it.n_kv && ok; ++j) {
          const int g = kvc + j, st = g % ST;
          if (!mbar_wait_warp(kv_full + st, (g / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
          const uint32_t k_addr = smem_u32(sKV + st * 2 * Cfg::kTile);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= (t == 0 ? it.nkv0 : it.nkv1)) continue;
            // S_t is free once the softmax has read the previous S_t
            if (cs[t] > 0 && !mbar_wait_warp(s_free + t, (cs[t] - 1) & 1, p.err, kErrAttnMma)) { ok = false; break; }
            tc_fence_after();
            const uint32_t qa = q_addr + t * Cfg::kTile;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
              const int atom = (ks * 16) / Cfg::kAtomCols;
              const int within = ((ks * 16) % Cfg::kAtomCols) * 2;
              const uint64_t ad = smem_desc(qa + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
              const uint64_t bd = smem_desc(k_addr + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
              umma_f16_ss_elect(tmem + Cfg::kColS + t * 128, ad, bd, idesc_qk, ks != 0);
            }
            umma_commit_elect(s_full + t);
            ++cs[t];
          }
          if (!ok) break;
          umma_commit_elect(kv_empty + st);  // K_j read once this warp's S MMAs retire
        }
        if (!ok) break;
        umma_commit_elect(q_empty + qb);  // both Q tiles read
        kvc += it.n_kv;
      }
    } else {
      // ------------------------------------------------------------ P.V issuer of query tile t
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, HD, false, true);
      const int t = warp - 10;
      const uint32_t o_tmem = tmem + Cfg::kColO + t * HD;
      const uint32_t p_tmem = tmem + Cfg::kColP + t * 64;
      int kvc = 0, cp = 0;  // cp: P_t consumed so far
      bool ok = true;
      for (int n = 0; ok; ++n) {
        int item;
        if (!next_item(n, item, kErrAttnMma) || item < 0) break;
        Item it;
        decode(item, it);
        const int nkv_t = t == 0 ? it.nkv0 : it.nkv1;
        for (int j = 0; j < it.n_kv; ++j) {
          const int g = kvc + j, st = g % ST;
          if (!mbar_wait_warp(kv_full + st, (g / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
          if (j >= nkv_t) {  // this tile is done with the item: release the stage as it lands
            mbar_arrive_elect(kv_empty + st);
            continue;
          }
          if (!mbar_wait_warp(p_full + t, cp & 1, p.err, kErrAttnMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sKV + st * 2 * Cfg::kTile) + Cfg::kTile;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t bd = smem_desc(v_addr + ks * 16 * Cfg::kRowB, Cfg::kAtomBytes, 8 * Cfg::kRowB, Cfg::kSw);
            umma_f16_ts_elect(o_tmem, p_tmem + ks * 8, bd, idesc_pv, (j | ks) != 0);
          }
          umma_commit_elect(pv_done + t);
          if (j == nkv_t - 1) umma_commit_elect(o_final + t);
          umma_commit_elect(kv_empty + st);
          ++cp;
        }
        kvc += it.n_kv;
      }
    }
  } else {
    reg_alloc<PC::kRegSoftmax>();
    // -------------------------------------------------------------- softmax + epilogue
    const int t = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + Cfg::kColS + t * 128;
    const uint32_t p_col = tmem + lane_off + Cfg::kColP + t * 64;
    const uint32_t o_col = tmem + lane_off + Cfg::kColO + t * HD;
    const float sl2 = p.scale_log2;
    // Normalise this thread's O row and store it as the fp16 context row.
    auto store_o = [&](__half* dst, float inv) {
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_col + c * 32, o);
        tmem_ld_wait();
        if (dst != nullptr) {
#pragma unroll
          for (int i2 = 0; i2 < 32; i2 += 8) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(o[i2]) * inv, __uint_as_float(o[i2 + 1]) * inv);
            w.y = pack_half2(__uint_as_float(o[i2 + 2]) * inv, __uint_as_float(o[i2 + 3]) * inv);
            w.z = pack_half2(__uint_as_float(o[i2 + 4]) * inv, __uint_as_float(o[i2 + 5]) * inv);
            w.w = pack_half2(__uint_as_float(o[i2 + 6]) * inv, __uint_as_float(o[i2 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + i2) = w;
          }
        }
      }
    };
    int cs = 0;  // S_t / P_t uses so far
    int co = 0;  // items of this tile drained so far
    bool pending = false;  // an item's O_t still waits in TMEM
    __half* prev_dst = nullptr;
    float prev_inv = 0.0f;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      int item;
      if (!next_item(n, item, kErrAttnSoftmax)) { ok = false; break; }
      if (item < 0) break;
      Item it;
      decode(item, it);
      const int nkv_t = t == 0 ? it.nkv0 : it.nkv1;
      if (nkv_t == 0) continue;
      const int qrow = (it.q0 + t) * 128 + r;
      const uint8_t* kmask = it.general ? p.mask + (size_t)it.b * p.S : nullptr;
      float m_run = -INFINITY, l_run = 0.0f;
      for (int j = 0; j < nkv_t; ++j) {
        const int u = cs + j;
        if (!mbar_wait(s_full + t, u & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[128];
        tmem_ld32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
        tmem_ld32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        tmem_ld32(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
        tmem_ld32(s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(s_free + t);  // S_t may now be overwritten
        const int kbase = j * 128;
        const bool diag = p.causal && j == it.qg0 + t;
        const bool tail = kbase + 128 > it.len;
        if (diag || tail) {
          const int lim_causal = diag ? r : 127;
          const int lim_len = it.len - kbase - 1;
          mask_past(s, lim_causal < lim_len ? lim_causal : lim_len);
        }
        if (kmask) mask_keys(s, kmask + kbase);
        const float mx = row_max128(s);
        const float m_tile = mx * sl2;
        const bool grow = m_tile > m_run + Cfg::kRescaleLog2;
        float alpha = 1.0f;
        if (grow) {
          alpha = fast_exp2(m_run - m_tile);  // 0 when m_run = -inf
          m_run = m_tile;
        }
        const float msub = m_run == -INFINITY ? 0.0f : m_run;
        const float rowsum = exp_pack_rowsum(s, sl2, msub);
        if (j == 0) {
          if (pending) {
            // the previous item's last P.V has retired: P_t is free and its O_t final
            if (!mbar_wait(o_final + t, co & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
            tc_fence_after();
            store_o(prev_dst, prev_inv);
            ++co;
            pending = false;
          }
        } else {
          // P_t and O_t are free once P.V_t(j-1) has retired
          if (!mbar_wait(pv_done + t, (u - 1) & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_st32(p_col, *reinterpret_cast<uint32_t(*)[32]>(s));
        tmem_st32(p_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        l_run = l_run * alpha + rowsum;
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(o_col + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i2 = 0; i2 < 32; ++i2) o[i2] = __float_as_uint(__uint_as_float(o[i2]) * alpha);
            tmem_st32(o_col + c * 32, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full + t);
      }
      if (!ok) break;
      cs += nkv_t;
      pending = true;
      prev_inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      const long long crow = ctx_row(p, it.b, qrow);
      prev_dst = crow >= 0 ? p.ctx + (size_t)crow * p.d_model + (size_t)it.h * HD : nullptr;
    }
    if (ok && pending && mbar_wait(o_final + t, co & 1, p.err, kErrAttnSoftmax)) {
      tc_fence_after();
      store_o(prev_dst, prev_inv);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, Cfg::kTmemCols);
  if (threadIdx.x == 0 && p.sched != nullptr) {
    // the last CTA out resets the scheduler for the next launch (every CTA's
    // producer has stopped claiming by the time it counts itself done)
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

}  // namespace tj
