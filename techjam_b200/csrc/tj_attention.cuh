// Flash-style causal / padded self-attention on tcgen05.
//
// One CTA per (128-query tile, head, sample).  Q, K, V are fp16 [B, H, S, HD]
// (written by the packed-QKV GEMM epilogue); the context is written fp16 into
// [B*S, d_model] at column h*HD so the output projection reads it directly.
//
//   warp 4      TMA producer: Q once, then K/V tiles into a STAGES-deep ring
//   warp 5      one thread issues S = Q K^T into TMEM (double-buffered) and,
//               one block behind, O_j = P_j V_j into TMEM (double-buffered)
//   warps 0..3  softmax: thread r owns query row r; reads S row from TMEM,
//               online softmax in fp32 (exp2 domain), writes P (fp16) to a
//               swizzled smem tile, accumulates O_j into registers with the
//               running-max correction, normalises at the end.
//
// Tile skipping: key tiles above the diagonal are never visited; query tiles
// past a sample's valid length exit at once; with causal + right padding the
// key mask is provably redundant (every key <= a valid query is valid) and is
// not evaluated.  Rows whose keys are all masked produce 0.
#pragma once
#include "tj_common.cuh"

namespace tj {

struct AttnParams {
  const int* lengths;   // [B]
  const uint8_t* mask;  // [B*S] key/row validity; used only for samples flagged general
  const uint8_t* general;  // [B] 1 if the sample's mask is not a right-padded prefix
  __half* ctx;          // [B*S, d_model]
  int S, H, d_model;
  int causal;
  float scale_log2;     // head_dim^-0.5 * log2(e)
  int* err;
};

template <int HD>
struct AttnCfg {
  static constexpr int kSw = HD >= 64 ? 128 : 64;      // swizzle span (bytes) of Q/K/V rows
  static constexpr int kRowB = kSw;                     // bytes per smem row inside one atom
  static constexpr int kAtomCols = kSw / 2;             // fp16 columns per atom
  static constexpr int kAtoms = HD / kAtomCols;
  static constexpr int kAtomBytes = 128 * kRowB;
  static constexpr int kTile = 128 * HD * 2;
  static constexpr int kStages = HD >= 128 ? 2 : 3;
  static constexpr int kPBytes = 128 * 128 * 2;
  static constexpr int kSmemBytes = kTile + kStages * 2 * kTile + 2 * kPBytes + 1024 + 256;
  static constexpr int kTmemCols = 512;
  static_assert(HD == 32 || HD == 64 || HD == 128, "head_dim must be 32, 64 or 128");
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<HD>;
  constexpr int ST = Cfg::kStages;
  const int bh = blockIdx.y;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int n_qt = gridDim.x;
  const int qt = p.causal ? (n_qt - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int len = __ldg(p.lengths + b);
  if (qt * 128 >= len) return;
  if (error_raised(p.err)) return;
  const bool general = p.mask != nullptr && __ldg(p.general + b) != 0;
  const int n_kv = p.causal ? (qt + 1) : (len + 127) / 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + Cfg::kTile;                      // stage s: K at s*2*kTile, V after it
  uint8_t* sP = sKV + ST * 2 * Cfg::kTile;            // [2][128 x 128] fp16
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < ST; ++i) { mbar_init(kv_full + i, 1); mbar_init(kv_empty + i, 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(s_full + i, 1); mbar_init(p_full + i, 128); mbar_init(o_full + i, 1); }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int row0 = bh * p.S;  // first row of this (b, h) in the [B*H*S, HD] views

  if (warp == 4) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_expect_tx(q_full, Cfg::kTile);
#pragma unroll
      for (int a = 0; a < Cfg::kAtoms; ++a)
        tma_load_2d(sQ + a * Cfg::kAtomBytes, &tmQ, q_full, a * Cfg::kAtomCols, row0 + qt * 128);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        if (!mbar_wait(kv_empty + st, ((j / ST) & 1) ^ 1, p.err, kErrAttnProducer)) break;
        uint8_t* sk = sKV + st * 2 * Cfg::kTile;
        uint8_t* sv = sk + Cfg::kTile;
        mbar_expect_tx(kv_full + st, 2 * Cfg::kTile);
#pragma unroll
        for (int a = 0; a < Cfg::kAtoms; ++a) {
          tma_load_2d(sk + a * Cfg::kAtomBytes, &tmK, kv_full + st, a * Cfg::kAtomCols, row0 + j * 128);
          tma_load_2d(sv + a * Cfg::kAtomBytes, &tmV, kv_full + st, a * Cfg::kAtomCols, row0 + j * 128);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_qk = idesc_f16_f32(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.err, kErrAttnMma);
      auto issue_pv = [&](int jj) -> bool {
        const int pb = jj & 1;
        if (!mbar_wait(p_full + pb, (jj >> 1) & 1, p.err, kErrAttnMma)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + pb * Cfg::kPBytes);
        const uint32_t v_addr = smem_u32(sKV + (jj % ST) * 2 * Cfg::kTile + Cfg::kTile);
        const uint32_t o_tmem = tmem + 256 + pb * HD;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t ad = smem_desc(p_addr + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, 128);
          const uint64_t bd = smem_desc(v_addr + ks * 16 * Cfg::kRowB, Cfg::kAtomBytes, 8 * Cfg::kRowB, Cfg::kSw);
          umma_f16_ss(o_tmem, ad, bd, idesc_pv, ks != 0);
        }
        umma_commit(o_full + pb);
        umma_commit(kv_empty + (jj % ST));
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % ST;
        if (!mbar_wait(kv_full + st, (j / ST) & 1, p.err, kErrAttnMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + st * 2 * Cfg::kTile);
        const uint32_t s_tmem = tmem + (j & 1) * 128;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const int atom = (ks * 16) / Cfg::kAtomCols;
          const int within = ((ks * 16) % Cfg::kAtomCols) * 2;
          const uint64_t ad = smem_desc(q_addr + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
          const uint64_t bd = smem_desc(k_addr + atom * Cfg::kAtomBytes + within, 16, 8 * Cfg::kRowB, Cfg::kSw);
          umma_f16_ss(s_tmem, ad, bd, idesc_qk, ks != 0);
        }
        umma_commit(s_full + (j & 1));
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n_kv >= 1) issue_pv(n_kv - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp;  // warps 0..3 own TMEM lanes 32*warp .. +31
    const int r = quarter * 32 + lane;
    const int qrow = qt * 128 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.0f, m_acc = -INFINITY;
    float m_hist[2] = {0.0f, 0.0f};
    float o_acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o_acc[i] = 0.0f;
    const uint8_t* kmask = general ? p.mask + (size_t)b * p.S : nullptr;
    bool ok = true;

    auto accumulate_o = [&](int jj, float m_ref) -> bool {
      const int ob = jj & 1;
      if (!mbar_wait(o_full + ob, (jj >> 1) & 1, p.err, kErrAttnSoftmax)) return false;
      tc_fence_after();
      const float f_old = exp2f(m_acc - m_ref);
      const float f_new = exp2f(m_hist[ob] - m_ref);
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + 256 + ob * HD + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o_acc[c * 32 + i] = o_acc[c * 32 + i] * f_old + __uint_as_float(o[i]) * f_new;
      }
      m_acc = m_ref;
      return true;
    };

    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(s_full + sb, (j >> 1) & 1, p.err, kErrAttnSoftmax)) { ok = false; break; }
      tc_fence_after();
      const int kbase = j * 128;
      const bool need_mask = general || (p.causal ? (j == qt) : (kbase + 128 > len));
      const uint32_t s_addr = lane_base + sb * 128;
      // pass 1: row max (log2-scaled)
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t s[32];
        tmem_ld32(s_addr + c * 32, s);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = __uint_as_float(s[i]) * sl2;
          if (need_mask) {
            const int key = kbase + c * 32 + i;
            const bool dead = (p.causal && key > qrow) || key >= len || (kmask && kmask[key] == 0);
            v = dead ? -INFINITY : v;
          }
          mx = fmaxf(mx, v);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
      const float alpha = exp2f(m_run - m_use);
      // the P buffer of this parity is free once PV_{j-2} retired; fold O_{j-2} in
      if (j >= 2 && !accumulate_o(j - 2, m_use)) { ok = false; break; }
      // pass 2: probabilities -> fp16 P tile (128B-swizzled, K-major)
      float rowsum = 0.0f;
      uint8_t* prow = sP + sb * Cfg::kPBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t s[32];
        tmem_ld32(s_addr + c * 32, s);
        tmem_ld_wait();
        float pv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = __uint_as_float(s[i]) * sl2;
          if (need_mask) {
            const int key = kbase + c * 32 + i;
            const bool dead = (p.causal && key > qrow) || key >= len || (kmask && kmask[key] == 0);
            v = dead ? -INFINITY : v;
          }
          pv[i] = exp2f(v - m_use);
          rowsum += pv[i];
        }
        uint8_t* atom = prow + (c >> 1) * 16384;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (c & 1) * 4 + q;
          uint4 w;
          w.x = pack_half2(pv[q * 8 + 0], pv[q * 8 + 1]);
          w.y = pack_half2(pv[q * 8 + 2], pv[q * 8 + 3]);
          w.z = pack_half2(pv[q * 8 + 4], pv[q * 8 + 5]);
          w.w = pack_half2(pv[q * 8 + 6], pv[q * 8 + 7]);
          *reinterpret_cast<uint4*>(atom + ((ch ^ (r & 7)) << 4)) = w;
        }
      }
      l_run = l_run * alpha + rowsum;
      m_run = m_new;
      m_hist[sb] = m_use;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full + sb);
    }
    if (ok) {
      const float m_ref = (m_run == -INFINITY) ? 0.0f : m_run;
      for (int jj = (n_kv >= 2 ? n_kv - 2 : 0); jj < n_kv && ok; ++jj) ok = accumulate_o(jj, m_ref);
    }
    if (ok && qrow < p.S) {
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      __half* dst = p.ctx + ((size_t)b * p.S + qrow) * p.d_model + (size_t)h * HD;
#pragma unroll
      for (int i = 0; i < HD; i += 8) {
        uint4 w;
        w.x = pack_half2(o_acc[i] * inv, o_acc[i + 1] * inv);
        w.y = pack_half2(o_acc[i + 2] * inv, o_acc[i + 3] * inv);
        w.z = pack_half2(o_acc[i + 4] * inv, o_acc[i + 5] * inv);
        w.w = pack_half2(o_acc[i + 6] * inv, o_acc[i + 7] * inv);
        *reinterpret_cast<uint4*>(dst + i) = w;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace tj
