// Warp-level selection helpers shared by the row top-k and the within-cluster top-q.
#pragma once
#include "oa_common.cuh"

namespace oa {

// ---- threshold + sort selection of the k largest unique 64-bit words held by a warp.  A word packs
// (key << 32) | (0xffffffff - index), so "larger" means larger key, ties to the lower index.  The
// k-th largest of the 32 lane maxima is a lower bound T0 of the answer (at least k words reach it);
// the words >= T0 are compacted (at most 64, else the caller falls back to the radix select) and
// sorted by a 64-element bitonic network in registers.
__device__ __forceinline__ uint64_t shfl64(uint64_t v, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
  const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
  return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl64_xor(uint64_t v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
  return ((uint64_t)hi << 32) | lo;
}
// descending bitonic sort of the 32 words v (one per lane)
__device__ __forceinline__ uint64_t bitonic32_desc(uint64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 1; j >>= 1) {
      const uint64_t o = shfl64_xor(v, j);
      const int l = lane ^ j;
      const bool keep_max = ((lane & k) == 0) == (lane < l);
      v = keep_max ? (o > v ? o : v) : (o < v ? o : v);
    }
  }
  return v;
}
// descending bitonic sort of 64 words: element e = lane + 32 h lives in v[h] of lane e & 31
__device__ __forceinline__ void bitonic64_desc(uint64_t (&v)[2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 1; j >>= 1) {
      if (j == 32) {  // partners in the same lane
        const bool keep_max = (lane & k) == 0;  // element lane (< lane + 32)
        const uint64_t a = v[0], b = v[1];
        v[0] = keep_max ? (a > b ? a : b) : (a < b ? a : b);
        v[1] = keep_max ? (a > b ? b : a) : (a < b ? b : a);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int e = lane + 32 * h;
          const uint64_t o = shfl64_xor(v[h], j);
          const bool keep_max = ((e & k) == 0) == (e < (e ^ j));
          v[h] = keep_max ? (o > v[h] ? o : v[h]) : (o < v[h] ? o : v[h]);
        }
      }
    }
  }
}
// Top k (k <= 32) of the m words word(i), i < m (0 = no word).  On success, sorted[0..1] hold the
// survivors (at most 64, at least k) in descending order (element e = lane + 32 h, 0 past the end)
// and kth the k-th largest.  Fails when more than 64 words survive or fewer than k words exist.
template <typename Word>
__device__ __forceinline__ bool warp_topk_sorted(int m, int k, Word word, uint64_t* sbuf, uint64_t (&sorted)[2],
                                                 uint64_t& kth) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  if (k < 1 || k > 32) return false;
  uint64_t lm = 0ull;
  for (int i = lane; i < m; i += 32) {
    const uint64_t w = word(i);
    lm = w > lm ? w : lm;
  }
  uint64_t T0 = shfl64(bitonic32_desc(lm), k - 1);
  if (T0 == 0ull) T0 = 1ull;  // fewer than k lanes hold words: every word survives
  int cnt = 0;
  for (int i0 = 0; i0 < m; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t w = i < m ? word(i) : 0ull;
    const unsigned b = __ballot_sync(0xffffffffu, w >= T0 && w != 0ull);
    if (w >= T0 && w != 0ull && cnt + __popc(b & lt) < 64) sbuf[cnt + __popc(b & lt)] = w;
    cnt += __popc(b);
  }
  if (cnt > 64 || cnt < k) return false;
  __syncwarp();
  sorted[0] = lane < cnt ? sbuf[lane] : 0ull;
  sorted[1] = lane + 32 < cnt ? sbuf[lane + 32] : 0ull;
  __syncwarp();
  bitonic64_desc(sorted);
  kth = shfl64(k > 32 ? sorted[1] : sorted[0], (k - 1) & 31);
  return true;
}

// ---- the same selection on 32-bit words ((16-bit key << 16) | (0xffff - index)), for keys that
// carry 16 bits of order and fewer than 65536 candidates: half the shuffles and compares
__device__ __forceinline__ uint32_t bitonic32_desc_u32(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 1; j >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool keep_max = ((lane & k) == 0) == (lane < (lane ^ j));
      v = keep_max ? max(o, v) : min(o, v);
    }
  }
  return v;
}
__device__ __forceinline__ void bitonic64_desc_u32(uint32_t (&v)[2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 1; j >>= 1) {
      if (j == 32) {  // partners in the same lane
        const bool keep_max = (lane & k) == 0;
        const uint32_t a = v[0], b = v[1];
        v[0] = keep_max ? max(a, b) : min(a, b);
        v[1] = keep_max ? min(a, b) : max(a, b);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int e = lane + 32 * h;
          const uint32_t o = __shfl_xor_sync(0xffffffffu, v[h], j);
          const bool keep_max = ((e & k) == 0) == (e < (e ^ j));
          v[h] = keep_max ? max(o, v[h]) : min(o, v[h]);
        }
      }
    }
  }
}
template <typename Word>
__device__ __forceinline__ bool warp_topk_sorted32(int m, int k, Word word, uint32_t* sbuf, uint32_t (&sorted)[2],
                                                   uint32_t& kth) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  if (k < 1 || k > 32) return false;
  uint32_t lm = 0u;
  for (int i = lane; i < m; i += 32) lm = max(lm, word(i));
  uint32_t T0 = __shfl_sync(0xffffffffu, bitonic32_desc_u32(lm), k - 1);
  if (T0 == 0u) T0 = 1u;  // fewer than k lanes hold words: every word survives
  int cnt = 0;
  for (int i0 = 0; i0 < m; i0 += 32) {
    const int i = i0 + lane;
    const uint32_t w = i < m ? word(i) : 0u;
    const bool s = w >= T0 && w != 0u;
    const unsigned b = __ballot_sync(0xffffffffu, s);
    if (s && cnt + __popc(b & lt) < 64) sbuf[cnt + __popc(b & lt)] = w;
    cnt += __popc(b);
  }
  if (cnt > 64 || cnt < k) return false;
  __syncwarp();
  sorted[0] = lane < cnt ? sbuf[lane] : 0u;
  sorted[1] = lane + 32 < cnt ? sbuf[lane + 32] : 0u;
  __syncwarp();
  bitonic64_desc_u32(sorted);
  kth = __shfl_sync(0xffffffffu, k > 32 ? sorted[1] : sorted[0], (k - 1) & 31);
  return true;
}

}  // namespace oa
