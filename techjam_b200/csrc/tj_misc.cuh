// Memory-bound helper kernels: mask -> lengths / live-tile list, LayerNorm,
// and the one-time weight packing (fp32 nn.Linear weights -> fp16).
#pragma once
#include "tj_common.cuh"

namespace tj {

constexpr int kTileRows = 128;

// Per sample: length = 1 + last valid position (0 if none); general = mask is
// not a right-padded prefix.  mask == null means every position is valid.
// sched (nullable): the attention scheduler's two words, zeroed here so that a
// forward starts from a clean scheduler even after an aborted launch.
// counts (nullable): valid tokens per sample.
__global__ void __launch_bounds__(1024) prep_lengths_kernel(const uint8_t* __restrict__ mask, int S,
                                                             int* __restrict__ lengths,
                                                             uint8_t* __restrict__ general, int* __restrict__ sched,
                                                             int* __restrict__ counts) {
  const int b = blockIdx.x;
  griddep_launch_dependents();
  griddep_wait();
  if (sched != nullptr && b == 0 && threadIdx.x < 2) sched[threadIdx.x] = 0;
  if (mask == nullptr) {
    if (threadIdx.x == 0) {
      lengths[b] = S;
      general[b] = 0;
      if (counts != nullptr) counts[b] = S;
    }
    return;
  }
  const uint8_t* m = mask + (size_t)b * S;
  int last = 0, count = 0;
  if ((S & 15) == 0 && (reinterpret_cast<uintptr_t>(m) & 15) == 0) {
    // 16 mask bytes per load; per byte: nonzero = valid
    const uint4* m16 = reinterpret_cast<const uint4*>(m);
    for (int i = threadIdx.x; i < S / 16; i += blockDim.x) {
      const uint4 w = m16[i];
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t nz = __vcmpne4(words[q], 0u);  // 0xff per valid byte
        count += __popc(nz) >> 3;
        if (nz) last = 16 * i + 4 * q + 4 - (__clz(nz) >> 3);
      }
    }
  } else {
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
      if (m[i]) { last = i + 1; ++count; }
    }
  }
  __shared__ int s_last[32], s_count[32];
  for (int o = 16; o > 0; o >>= 1) {
    last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    count += __shfl_xor_sync(0xffffffffu, count, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { s_last[w] = last; s_count[w] = count; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    last = l < nw ? s_last[l] : 0;
    count = l < nw ? s_count[l] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
      count += __shfl_xor_sync(0xffffffffu, count, o);
    }
    if (l == 0) {
      lengths[b] = last;
      general[b] = (count != last) ? 1 : 0;
      if (counts != nullptr) counts[b] = count;
    }
  }
}

// Compact list of 128-row tiles (over the flattened [B*S] rows) holding at
// least one row inside its sample's valid prefix.  One block of 1024 threads.
__global__ void prep_tiles_kernel(const int* lengths, int B, int S, int* __restrict__ tile_list,
                                  int* __restrict__ n_live, uint8_t* __restrict__ tile_live) {
  griddep_launch_dependents();
  griddep_wait();
  const long long M = (long long)B * S;
  const int n_tiles = (int)((M + kTileRows - 1) / kTileRows);
  __shared__ int s_warp[32];
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int start = 0; start < n_tiles; start += blockDim.x) {
    const int t = start + threadIdx.x;
    int live = 0;
    if (t < n_tiles) {
      const long long r0 = (long long)t * kTileRows;
      const long long r1 = min(r0 + kTileRows, M) - 1;
      for (long long b = r0 / S; b <= r1 / S; ++b) {
        const long long first = max(r0, b * S) - b * S;
        if (first < lengths[b]) { live = 1; break; }
      }
      tile_live[t] = (uint8_t)live;
    }
    // block-wide exclusive scan of `live`
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    int incl = live;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (l >= o) incl += v;
    }
    if (l == 31) s_warp[w] = incl;
    __syncthreads();
    if (w == 0) {
      int v = s_warp[l];
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (l >= o) v += u;
      }
      s_warp[l] = v;
    }
    __syncthreads();
    const int excl = incl - live + (w > 0 ? s_warp[w - 1] : 0);
    if (live) tile_list[s_base + excl] = t;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_base += excl + live;
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_live = s_base;
}

// Varlen token packing: the valid tokens of the [B*S] rows, sample by sample
// in position order, become packed rows 0..T_v-1.  One block per sample:
// pack_of[b*S + n] = packed row of token (b, n) or -1; row_of[packed] = b*S + n.
// A right-padded sample's tokens are its first lengths[b] positions; a
// general mask's are found with a block-wide scan.
__global__ void __launch_bounds__(1024) prep_pack_kernel(const uint8_t* __restrict__ mask, int S,
                                                          const int* lengths, const uint8_t* general,
                                                          const int* counts, int* __restrict__ pack_of,
                                                          int* __restrict__ row_of) {
  const int b = blockIdx.x;
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int s_warp[32];
  __shared__ int s_off, s_base;
  // exclusive prefix of the earlier samples' token counts
  int part = 0;
  for (int i = threadIdx.x; i < b; i += blockDim.x) part += counts[i];
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (l == 0) s_warp[w] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += s_warp[i];
    s_off = t;
    s_base = 0;
  }
  __syncthreads();
  const int off = s_off;
  const long long row0 = (long long)b * S;
  if (mask == nullptr || general[b] == 0) {
    const int len = lengths[b];
    for (int n = threadIdx.x; n < S; n += blockDim.x) {
      const int k = n < len ? off + n : -1;
      pack_of[row0 + n] = k;
      if (k >= 0) row_of[k] = (int)(row0 + n);
    }
    return;
  }
  for (int start = 0; start < S; start += blockDim.x) {
    __syncthreads();  // s_warp reuse
    const int n = start + threadIdx.x;
    const int v = n < S && mask[row0 + n] != 0 ? 1 : 0;
    int incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (l >= o) incl += u;
    }
    if (l == 31) s_warp[w] = incl;
    __syncthreads();
    if (w == 0) {
      int x = s_warp[l];
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += u;
      }
      s_warp[l] = x;
    }
    __syncthreads();
    const int excl = incl - v + (w > 0 ? s_warp[w - 1] : 0);
    if (n < S) {
      const int k = v ? off + s_base + excl : -1;
      pack_of[row0 + n] = k;
      if (k >= 0) row_of[k] = (int)(row0 + n);
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_base += excl + v;
  }
}

// Live tiles of the packed rows: tiles 0 .. ceil(T_v/128)-1, and row_of = -1
// for the packed rows of the last tile past T_v.  One block.
__global__ void prep_pack_tiles_kernel(const int* counts, int B, int* __restrict__ row_of,
                                       int* __restrict__ tile_list, int* __restrict__ n_live,
                                       uint8_t* __restrict__ tile_live, int n_tiles_all) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int s_warp[32];
  int part = 0;
  for (int i = threadIdx.x; i < B; i += blockDim.x) part += counts[i];
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = part;
  __syncthreads();
  int tv = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tv += s_warp[i];
  const int tiles = (tv + kTileRows - 1) / kTileRows;
  for (int t = threadIdx.x; t < n_tiles_all; t += blockDim.x) {
    tile_list[t] = t;
    tile_live[t] = t < tiles ? 1 : 0;
  }
  for (int r = tv + (int)threadIdx.x; r < tiles * kTileRows; r += blockDim.x) row_of[r] = -1;
  if (threadIdx.x == 0) *n_live = tiles;
}

// Row addressing of the LayerNorm kernels: padded row r is token (r / S,
// r % S), valid inside the sample's prefix (and its mask).  Its output row is
// r, or pack_of[r] with varlen packing (then invalid rows are not written).
struct RowValidity {
  const int* lengths;
  const uint8_t* mask;
  int S;
  long long M;
  const int* pack_of;
  __device__ bool operator()(long long row) const {
    if (row >= M) return false;
    const int b = (int)(row / S);
    const int n = (int)(row - (long long)b * S);
    if (n >= lengths[b]) return false;
    return mask == nullptr || __ldg(mask + row) != 0;
  }
};

// One warp per row, d <= 32*4*VPL.  Valid rows: (x-mean)/sqrt(var+eps)*g+b.
// Invalid rows inside live tiles (or every invalid row when ALL_ROWS) are
// written as zeros; rows of dead tiles are skipped.
template <int VPL, bool OUT_F16, bool ALL_ROWS>
__global__ void __launch_bounds__(256) layernorm_kernel(const float* x, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, void* __restrict__ out,
                                                        int d, float eps, RowValidity valid,
                                                        const uint8_t* tile_live) {
  griddep_launch_dependents();
  griddep_wait();
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= valid.M) return;
  const bool ok = valid(row);
  if (!ok && (valid.pack_of != nullptr || (!ALL_ROWS && tile_live[row / kTileRows] == 0))) return;
  // output row: issued now, used only by the stores at the end
  const long long orow = valid.pack_of != nullptr ? (long long)valid.pack_of[row] : row;
  const int nvec = d >> 2;
  float4 v[VPL];
  if (ok) {
    const float4* src = reinterpret_cast<const float4*>(x + row * d);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < nvec ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / d;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
        sq += (a * a + bb * bb) + (cc * cc + dd * dd);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / d + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
        const float4 bt = __ldg(reinterpret_cast<const float4*>(beta) + c);
        v[i].x = (v[i].x - mean) * rstd * g.x + bt.x;
        v[i].y = (v[i].y - mean) * rstd * g.y + bt.y;
        v[i].z = (v[i].z - mean) * rstd * g.z + bt.z;
        v[i].w = (v[i].w - mean) * rstd * g.w + bt.w;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      if constexpr (OUT_F16) {
        uint2 w;
        w.x = pack_half2(v[i].x, v[i].y);
        w.y = pack_half2(v[i].z, v[i].w);
        reinterpret_cast<uint2*>(static_cast<__half*>(out) + orow * d)[c] = w;
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(out) + orow * d)[c] = v[i];
      }
    }
  }
}

// Failure-path self-test: one warp waits, through the same bounded wait every
// kernel uses, on an mbarrier that nothing arrives at.  The wait runs out
// after the device's wait limit, records kErrTest in *err and the kernel
// returns -- no fault, trap or hang, and the context stays usable.
__global__ void wait_selftest_kernel(int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  mbar_wait_warp(&bar, 0, err, kErrTest);
}

// dst = fp16(src), element-wise, for the packed weight buffers.
__global__ void f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}

}  // namespace tj
