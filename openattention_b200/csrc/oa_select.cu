// Per-step selection front half on sm_100a: index update of the new token (+ the QGS query
// projection), the QGS scan over the int8 key codes, and the exact row top-k.
//
// Index update restates _k_index_update_d2 (inference/ours_graph.py:43-90); the query projection is
// methods_eager.py:603; the scan restates _k_qgs_scan_tm (inference/graph_runner.py:100-120) and the
// top-k _k_select (inference/graph_runner.py:123-159).
//
// QGS scores are computed EXACTLY with int8 tensor-core MMAs: each query head's zq (32 bf16 values)
// is mapped to integers Z_j = trunc(z_j * 2^S), S = 29 - e_max, |Z_j| < 2^30, split into four signed
// 8-bit limbs; one mma.m16n8k32.s8 multiplies 16 tokens' codes by 8 (head, limb) columns, and the
// limb partial sums recombine into the exact int64 dot product, which is rounded once to fp32 and
// once to bf16.  The result does not depend on summation order.
#include "oa_common.cuh"
#include "oa_warp.cuh"
#include "../../include/openattention_b200.h"

namespace oa {
namespace {

// ------------------------------------------------------------------------ index update (+ zq)
struct IndexArgs {
  const __nv_bfloat16* K;
  const __nv_bfloat16* V;
  int8_t* codes;
  const float* U;
  const float* scale;
  const __nv_bfloat16* W;
  const float* colmean;
  const float* cent;
  int32_t* asg;
  float* nb;
  float* Sk;
  float* Sk2;
  float* Sv;
  int32_t* reclist;
  int32_t* reccnt;
  int rmax;
  const __nv_bfloat16* q;
  int64_t q_stride;
  __nv_bfloat16* zq;
  const int32_t* n_dev;
  int Lmax, C;
  // optional: the new token's K / V rows (B*8, 128) bf16; the key and value are taken from here and
  // the first query head's CTA of each KV head writes them into K / V at position n - 1
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
};

// One CTA per QUERY head r = kv*4 + g (so a batch's whole index update is resident at once): the
// KV head's QGS basis U, this head's QGC projection W and centroids are staged together; warp 0
// forms zq for this head, warp 1 (g == 0 only) the KV head's code of the new key, warp 2 the rank-16
// projection zp; the four warps then score the centroids (ties -> lower cluster id) and the CTA
// updates the cluster's pooled sums.  Every dot keeps its sequential fma order over d (or c).
constexpr int kIuCentCache = 256;  // clusters whose centroids are staged in shared memory

__global__ void __launch_bounds__(128, 8) index_update_kernel(const IndexArgs a) {
  extern __shared__ __align__(16) float iu_cent[];  // min(C, kIuCentCache) x 16
  const int r = blockIdx.x;
  const int kv = r / kG, g = r % kG;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = __ldg(a.n_dev) - 1;
  __shared__ __align__(16) float kf[kD], vf[kD], qf[kD], zp[kRC];
  __shared__ __align__(16) float sU[kD * kRQ];              // this KV head's QGS basis
  __shared__ __align__(16) __nv_bfloat16 sW[kD * kRC];      // this query head's QGC projection
  __shared__ float s_bv[4];
  __shared__ int s_bi[4];
  const bool have_tok = pos >= 0 && pos < a.Lmax;
  const int C = a.C;
  const int cstage = min(C, kIuCentCache);
  const float* ce = a.cent + (int64_t)r * C * kRC;
  const float* Uk = a.U + (int64_t)kv * kD * kRQ;
  // U, W and the centroids go to shared memory as 16-byte asynchronous copies, issued together with
  // the loads of the new K / V element and q, so the staging costs one memory round trip and holds no
  // registers (8 CTAs of 128 threads per SM: every row of a 32-request batch is resident at once).
  constexpr int kUV = kD * kRQ / 4 / 128;  // float4 of U per thread (8)
  constexpr int kWV = kD * kRC / 8 / 128;  // uint4 of W per thread (2)
  const int ncv = cstage * kRC / 4;
#pragma unroll
  for (int u = 0; u < kUV; ++u)
    cp_async16(reinterpret_cast<float4*>(sU) + tid + 128 * u, reinterpret_cast<const float4*>(Uk) + tid + 128 * u);
#pragma unroll
  for (int u = 0; u < kWV; ++u)
    cp_async16(reinterpret_cast<uint4*>(sW) + tid + 128 * u,
               reinterpret_cast<const uint4*>(a.W + (int64_t)r * kD * kRC) + tid + 128 * u);
  // centroid row i's four 16-byte chunks k land at chunk k ^ ((i >> 1) & 3): the scoring's 16-byte
  // reads (one row per lane) then meet no bank conflicts
  for (int i = tid; i < ncv; i += 128)
    cp_async16(reinterpret_cast<float4*>(iu_cent) + (i & ~3) + ((i & 3) ^ ((i >> 3) & 3)),
               reinterpret_cast<const float4*>(ce) + i);
  __nv_bfloat16 kb = __float2bfloat16_rn(0.f), vb = kb, qb = kb;
  if (have_tok) {
    if (a.k_new != nullptr) {
      kb = a.k_new[(int64_t)kv * kD + tid];
      vb = a.v_new[(int64_t)kv * kD + tid];
      if (g == 0) {  // the cache write of the fused append (read again only by later kernels)
        const_cast<__nv_bfloat16*>(a.K)[((int64_t)kv * a.Lmax + pos) * kD + tid] = kb;
        const_cast<__nv_bfloat16*>(a.V)[((int64_t)kv * a.Lmax + pos) * kD + tid] = vb;
      }
    } else {
      kb = a.K[((int64_t)kv * a.Lmax + pos) * kD + tid];
      vb = a.V[((int64_t)kv * a.Lmax + pos) * kD + tid];
    }
  }
  if (a.q != nullptr) qb = a.q[(int64_t)r * a.q_stride + tid];
  cp_async_wait_all();
  kf[tid] = __bfloat162float(kb);
  vf[tid] = __bfloat162float(vb);
  qf[tid] = __bfloat162float(qb);
  __syncthreads();
  if (warp == 0) {  // query projection zq[r, j] = bf16((q . U[:, j]) * scale_j), d ascending
    if (a.q != nullptr) {
      const int j = lane;
      float acc = 0.f;
#pragma unroll 2
      for (int d = 0; d < kD; d += 4) {  // q four at a time (one broadcast 16-byte read), d ascending
        const float4 q4 = *reinterpret_cast<const float4*>(&qf[d]);
        acc = __fmaf_rn(q4.x, sU[d * kRQ + j], acc);
        acc = __fmaf_rn(q4.y, sU[(d + 1) * kRQ + j], acc);
        acc = __fmaf_rn(q4.z, sU[(d + 2) * kRQ + j], acc);
        acc = __fmaf_rn(q4.w, sU[(d + 3) * kRQ + j], acc);
      }
      a.zq[(int64_t)r * kRQ + j] = __float2bfloat16_rn(__fmul_rn(acc, __ldg(&a.scale[kv * kRQ + j])));
    }
  } else if (warp == 1) {  // QGS code of the new key (per KV head: query head 0 of the group writes it)
    if (have_tok && g == 0) {
      const int j = lane;
      float acc = 0.f;
#pragma unroll 2
      for (int d = 0; d < kD; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&kf[d]);
        acc = __fmaf_rn(k4.x, sU[d * kRQ + j], acc);
        acc = __fmaf_rn(k4.y, sU[(d + 1) * kRQ + j], acc);
        acc = __fmaf_rn(k4.z, sU[(d + 2) * kRQ + j], acc);
        acc = __fmaf_rn(k4.w, sU[(d + 3) * kRQ + j], acc);
      }
      float c = rintf(__fdiv_rn(acc, __ldg(&a.scale[kv * kRQ + j])));
      c = fminf(fmaxf(c, -127.f), 127.f);
      a.codes[((int64_t)kv * a.Lmax + pos) * kRQ + j] = (int8_t)c;
    }
  } else if (warp == 2) {  // rank-16 QGC projection: zp = bf16(k . W) - colmean
    if (have_tok && lane < kRC) {
      const int c = lane;
      float acc = 0.f;
#pragma unroll 2
      for (int d = 0; d < kD; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&kf[d]);
        acc = __fmaf_rn(k4.x, __bfloat162float(sW[d * kRC + c]), acc);
        acc = __fmaf_rn(k4.y, __bfloat162float(sW[(d + 1) * kRC + c]), acc);
        acc = __fmaf_rn(k4.z, __bfloat162float(sW[(d + 2) * kRC + c]), acc);
        acc = __fmaf_rn(k4.w, __bfloat162float(sW[(d + 3) * kRC + c]), acc);
      }
      zp[c] = __fsub_rn(bf_round(acc), __ldg(&a.colmean[r * kRC + c]));
    }
  }
  if (!have_tok) return;
  __syncthreads();
  // nearest centroid: thread i scores clusters i, i + 128, ...; ties -> lower cluster id
  float bestv = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = tid; i < C; i += 128) {
    float dot = 0.f, nrm = 0.f;
#pragma unroll
    for (int k = 0; k < kRC / 4; ++k) {  // chunk k of row i, c = 4k .. 4k + 3 ascending
      const float4 x4 = i < cstage ? reinterpret_cast<const float4*>(iu_cent)[i * 4 + (k ^ ((i >> 1) & 3))]
                                   : __ldg(reinterpret_cast<const float4*>(ce) + i * 4 + k);
      const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dot = __fmaf_rn(zp[4 * k + e], xs[e], dot);
        nrm = __fmaf_rn(xs[e], xs[e], nrm);
      }
    }
    const float dist = __fsub_rn(dot, __fmul_rn(0.5f, nrm));
    if (dist > bestv) {
      bestv = dist;
      besti = i;
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bestv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, off);
    if (ov > bestv || (ov == bestv && oi < besti)) {
      bestv = ov;
      besti = oi;
    }
  }
  if (lane == 0) {
    s_bv[warp] = bestv;
    s_bi[warp] = besti;
  }
  __syncthreads();
  bestv = s_bv[0];
  besti = s_bi[0];
#pragma unroll
  for (int w = 1; w < 4; ++w) {
    if (s_bv[w] > bestv || (s_bv[w] == bestv && s_bi[w] < besti)) {
      bestv = s_bv[w];
      besti = s_bi[w];
    }
  }
  const int cid = besti == 0x7fffffff ? 0 : besti;
  const int64_t row = (int64_t)r * C + cid;
  {  // one round-to-nearest add per element: a reduction without a return is the same value, no wait
    const int d = tid;
    atomicAdd(&a.Sk[row * kD + d], kf[d]);
    atomicAdd(&a.Sk2[row * kD + d], __fmul_rn(kf[d], kf[d]));
    atomicAdd(&a.Sv[row * kD + d], vf[d]);
  }
  if (tid == 0) {
    a.asg[(int64_t)r * a.Lmax + pos] = cid;
    atomicAdd(&a.nb[row], 1.f);
    if (a.reclist != nullptr) {
      const int cnt = a.reccnt[row];
      if (cnt < a.rmax) a.reclist[row * a.rmax + cnt] = pos;
      a.reccnt[row] = cnt + 1;
    }
  }
}

// ------------------------------------------------------------------------ QGS scan (int8 MMA)
constexpr int kTile = 256;         // tokens per CTA step (8 warps x 32 tokens)
constexpr int kMaxTile = 32;       // tokens per tile maximum (one warp's share of a step)
constexpr int kScanThreads = 256;
constexpr int kTilesPerCta = 3;  // 24 KB of codes: 8 CTAs (64 warps) per SM at 30 registers

struct ScanArgs {
  const int8_t* codes;
  const __nv_bfloat16* zq;
  const int32_t* n_dev;
  int ns, nl;
  int Lmax, NT;
  uint16_t* scores;  // bf16 bits (R, sw)
  int64_t sw;
  float* tmax;  // (R, tm_stride)
  int64_t tm_stride;
  int32_t* status;  // set to 1 if a bulk copy did not complete (may be null)
};

__device__ __forceinline__ float pow2f_exact(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }
__device__ __forceinline__ float scale_pow2(float x, int k) {
  while (k > 100) { x = __fmul_rn(x, pow2f_exact(100)); k -= 100; }
  while (k < -100) { x = __fmul_rn(x, pow2f_exact(-100)); k += 100; }
  return __fmul_rn(x, pow2f_exact(k));
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__global__ void __launch_bounds__(kScanThreads, 8) qgs_scan_kernel(const ScanArgs a) {
  const int kv = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int n = __ldg(a.n_dev);
  __shared__ __align__(128) int8_t sbuf[kTilesPerCta * kTile * kRQ];  // the CTA's codes chunk (24 KB)
  __shared__ __align__(8) uint64_t mbar[kTilesPerCta];  // one per 256-token tile of the chunk
  __shared__ int8_t limb[kG][4][kRQ];  // [head][limb][j]
  __shared__ int sS[kG];
  const int t_begin = blockIdx.y * kTilesPerCta;
  const int tok0 = t_begin * kTile;
  const int ntok = max(0, min(min(a.Lmax, n), tok0 + kTilesPerCta * kTile) - tok0);  // tokens to fetch
  if (tid == 0)
    for (int ti = 0; ti < kTilesPerCta; ++ti) mbar_init(smem_u32(&mbar[ti]));
  __syncthreads();
  // one bulk copy (TMA, no multicast) per 256-token tile, each on its own barrier, so the first tile's
  // MMAs start while the later tiles are still arriving
  if (tid == 0)
    for (int ti = 0; ti < kTilesPerCta && ti * kTile < ntok; ++ti)
      bulk_load(sbuf + ti * kTile * kRQ, a.codes + ((int64_t)kv * a.Lmax + tok0 + ti * kTile) * kRQ,
                (uint32_t)min(kTile, ntok - ti * kTile) * kRQ, smem_u32(&mbar[ti]));
  // fixed-point image of each head's zq (one warp per head), overlapping the copy
  if (warp < kG) {
    const float z = __bfloat162float(a.zq[(int64_t)(kv * kG + warp) * kRQ + lane]);
    float amax = fabsf(z);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const int e_max = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127;
    int S = 0, Z = 0;
    if (amax != 0.f && e_max >= -100) {
      S = 29 - e_max;
      Z = __float2int_rz(scale_pow2(z, S));
    }
    const int l0 = (int)(int8_t)(Z & 0xff);
    const int z1 = (Z - l0) >> 8;
    const int l1 = (int)(int8_t)(z1 & 0xff);
    const int z2 = (z1 - l1) >> 8;
    const int l2 = (int)(int8_t)(z2 & 0xff);
    const int l3 = (z2 - l2) >> 8;
    limb[warp][0][lane] = (int8_t)l0;
    limb[warp][1][lane] = (int8_t)l1;
    limb[warp][2][lane] = (int8_t)l2;
    limb[warp][3][lane] = (int8_t)l3;
    if (lane == 0) sS[warp] = S;
  }
  __syncthreads();
  // B fragments of the two MMAs: column n = gid -> head gid / 2, limb 2m + gid % 2 (m = 0: limbs 0-1,
  // m = 1: limbs 2-3); rows k = tig*4..+3 and 16 + tig*4..+3.  The accumulators of thread (gid, tig)
  // then hold all four limbs of head tig for tokens gid and gid + 8: no exchange between lanes.
  uint32_t bf[2][2];
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int h = gid >> 1, k = 2 * m + (gid & 1);
    bf[m][0] = *reinterpret_cast<const uint32_t*>(&limb[h][k][tig * 4]);
    bf[m][1] = *reinterpret_cast<const uint32_t*>(&limb[h][k][16 + tig * 4]);
  }
  const int S_h = sS[tig];
  const bool one_mul = S_h >= -100 && S_h <= 100;  // 2^-S is a normal float: one exact multiply
  const float inv2S = one_mul ? pow2f_exact(-S_h) : 0.f;
  uint16_t* srow = a.scores + (int64_t)(kv * kG + tig) * a.sw;
  bool failed = false;  // a tile's copy did not complete in the bounded wait (this warp stops computing)
  // exact limb sum l0 + l1 2^8 + l2 2^16 + l3 2^24 (|l| < 2^19) -> fp32 (one rounding) -> x 2^-S; the
  // caller rounds two of them to bf16 with one packed conversion
  auto finish = [&](int l0, int l1, int l2, int l3) -> float {
    const long long tot = (long long)(l3 * 256 + l2) * 65536 + (long long)(l1 * 256 + l0);
    const float f0 = __ll2float_rn(tot);
    return one_mul ? __fmul_rn(f0, inv2S) : scale_pow2(f0, -S_h);
  };
  const int nv = min(n, a.Lmax);  // positions with a score; the rest of a touched tile is written -inf
#pragma unroll
  for (int ti = 0; ti < kTilesPerCta; ++ti) {
    const int tile = t_begin + ti;
    const int t0 = tile * kTile;
    __nv_bfloat162 hmax2 = __floats2bfloat162_rn(-INFINITY, -INFINITY);  // head tig, this warp's 32 tokens
    if (!failed && t0 < n && t0 < a.Lmax) {
      failed = !__all_sync(0xffffffffu, mbar_wait(smem_u32(&mbar[ti]), 0));
      if (failed && lane == 0 && a.status != nullptr) atomicExch(a.status, 1);
    }
    if (!failed && t0 < n && t0 < a.Lmax) {
      // only the tiles holding sink / local positions or the end of the row test positions one by one
      const bool edge = t0 < a.ns || t0 + kTile > nv - a.nl;
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int lt0 = ti * kTile + warp * 32 + grp * 16;  // chunk-local first token of the 16
        const int ta = tok0 + lt0 + gid;
        // ldmatrix x4: matrices (rows 0-7 | 8-15) x (bytes 0-15 | 16-31) of the 16 x 32-byte tile
        uint32_t af[4];
        const int mi = lane >> 3, ri = lane & 7;
        const int8_t* rowp = sbuf + (lt0 + (mi & 1) * 8 + ri) * kRQ + (mi >> 1) * 16;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(af[0]), "=r"(af[1]), "=r"(af[2]), "=r"(af[3])
                     : "r"(smem_u32(rowp)));
        int d0[4], d1[4];
        mma_s8(d0, af, bf[0][0], bf[0][1]);
        mma_s8(d1, af, bf[1][0], bf[1][1]);
        // tokens ta (low half) and ta + 8 (high half) as one bf16 pair
        __nv_bfloat162 pk2 = __floats2bfloat162_rn(finish(d0[0], d0[1], d1[0], d1[1]), finish(d0[2], d0[3], d1[2], d1[3]));
        uint32_t pk = *reinterpret_cast<uint32_t*>(&pk2);
        if (edge) {
          uint32_t s0 = pk & 0xffffu, s1 = pk >> 16;
          if (ta < a.ns || ta >= n - a.nl || ta >= nv) s0 = 0xff80u;
          if (ta + 8 < a.ns || ta + 8 >= n - a.nl || ta + 8 >= nv) s1 = 0xff80u;
          if (ta < a.Lmax) srow[ta] = (uint16_t)s0;
          if (ta + 8 < a.Lmax) srow[ta + 8] = (uint16_t)s1;
          pk = s0 | (s1 << 16);
          pk2 = *reinterpret_cast<__nv_bfloat162*>(&pk);
        } else {
          // pair tokens with the neighbouring lane (gid ^ 1, same head): even gid stores tokens
          // (ta, ta + 1), odd gid tokens (ta + 7, ta + 8), each as one 4-byte store
          const uint32_t other = __shfl_xor_sync(0xffffffffu, pk, 4);
          if ((gid & 1) == 0)
            *reinterpret_cast<uint32_t*>(srow + ta) = (pk & 0xffffu) | (other << 16);
          else
            *reinterpret_cast<uint32_t*>(srow + ta + 7) = (other >> 16) | (pk & 0xffff0000u);
        }
        hmax2 = __hmax2(hmax2, pk2);  // exact: the maximum of bf16 values
      }
    }
    // maximum of this warp's 32 tokens for head tig (a 32-token tile): reduce over gid
    const int wt = tile * (kTile / kMaxTile) + warp;  // 32-token tile index
    float hmax = fmaxf(__low2float(hmax2), __high2float(hmax2));
    hmax = fmaxf(hmax, __shfl_xor_sync(0xffffffffu, hmax, 4));
    hmax = fmaxf(hmax, __shfl_xor_sync(0xffffffffu, hmax, 8));
    hmax = fmaxf(hmax, __shfl_xor_sync(0xffffffffu, hmax, 16));
    if (!failed && wt < a.NT && gid == 0) a.tmax[(int64_t)(kv * kG + tig) * a.tm_stride + wt] = hmax;
  }
  if (failed && lane == 0)  // leave no copy in flight: each wait is bounded and returns at once if done
    for (int ti = 0; ti < kTilesPerCta && ti * kTile < ntok; ++ti) mbar_wait(smem_u32(&mbar[ti]), 0);
}

// ------------------------------------------------------------------------ exact row top-k
// One warp per row.  (1) the kt2 = min(2k, tiles) tiles with the largest maxima (ties -> lower
// tile) by a warp radix select over the 32-bit float keys of the tile maxima; (2) the k largest
// scores inside those tiles (ties -> lower position) by a radix select over 16-bit score keys;
// (3) the k winners ranked by (score desc, position asc).
constexpr int kSelWarps = 4;
constexpr int kMaxKT2 = 128;

struct SelectArgs {
  uint16_t* scores;
  int64_t sw;
  const float* tmax;
  int64_t tm_stride;
  const int32_t* n_dev;
  int R, ns, nl, k_top, NT, Lmax;
  int32_t* sel;
  int NT_pad, kt2_max;  // shared-memory slots per warp: tile keys, candidate tiles
};

__device__ __forceinline__ uint32_t fkey(float x) {  // ascending float -> ascending uint32
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint32_t ukey16(uint32_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }

// The q-th largest key among the valid keys get(i), i < m (warp-collective).  Returns the
// threshold T and `above` = number of valid keys > T; if fewer than q keys are valid, T = 0 and
// above = the valid count.  Digits of 8 bits from the top; hist: 256 ints of warp-private smem.
template <int BITS, typename Get>
__device__ __forceinline__ void warp_radix_select(int m, int q, int* hist, Get get, uint32_t& T, int& above) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0u, pmask = 0u;
  above = 0;
  bool ok = true;
#pragma unroll 1
  for (int shift = BITS - 8; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    for (int i = lane; i < m; i += 32) {
      bool v;
      uint32_t k;
      get(i, v, k);
      if (v && (k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1);
    }
    __syncwarp();
    int cnt[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cnt[i] = hist[255 - 8 * lane - i];
      sum += cnt[i];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    const int excl = incl - sum;
    const int need = q - above;
    int fd = -1, fa = 0;
    if (excl < need && incl >= need) {
      int run = excl;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (fd < 0 && run + cnt[i] >= need) {
          fd = 255 - 8 * lane - i;
          fa = run;
        }
        run += cnt[i];
      }
    }
    const unsigned who = __ballot_sync(0xffffffffu, fd >= 0);
    __syncwarp();
    if (who == 0u) {  // fewer than q valid keys: take them all
      ok = false;
      above += __shfl_sync(0xffffffffu, incl, 31);
      break;
    }
    const int src = __ffs(who) - 1;
    const int d = __shfl_sync(0xffffffffu, fd, src);
    above += __shfl_sync(0xffffffffu, fa, src);
    prefix |= (uint32_t)d << shift;
    pmask |= 0xffu << shift;
  }
  T = ok ? prefix : 0u;
}

__global__ void __launch_bounds__(kSelWarps * 32) qgs_select_kernel(const SelectArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kSelWarps + warp;
  __shared__ int s_hist[kSelWarps][256];
  __shared__ int s_tiles[kSelWarps][kMaxKT2];
  __shared__ int s_pos[kSelWarps][64];
  __shared__ uint32_t s_key[kSelWarps][64];
  __shared__ uint64_t s_w64[kSelWarps][64];
  extern __shared__ __align__(16) unsigned char sel_smem[];
  // per warp: tile keys (NT uint32), then candidate keys (kt2_max * 256 uint16)
  uint32_t* tkey = reinterpret_cast<uint32_t*>(sel_smem) + (size_t)warp * a.NT_pad;
  uint16_t* ckey = reinterpret_cast<uint16_t*>(reinterpret_cast<uint32_t*>(sel_smem) + (size_t)kSelWarps * a.NT_pad) +
                   (size_t)warp * a.kt2_max * kMaxTile;
  if (r >= a.R) return;
  int* hist = s_hist[warp];
  int* tiles = s_tiles[warp];
  const int n = __ldg(a.n_dev);
  const int ntv = min(a.NT, (n + kMaxTile - 1) / kMaxTile);
  const int kt2 = min(2 * a.k_top, ntv);
  const float* tm = a.tmax + (int64_t)r * a.tm_stride;
  uint16_t* srw = a.scores + (int64_t)r * a.sw;
  uint32_t low16 = 0u;  // the OR of the maxima's low 16 bits
  {  // tile keys: the row's maxima with 16-byte loads, all of a lane's loads issued before its stores
    const int h = min(ntv, (int)((4u - ((uint32_t)(reinterpret_cast<uintptr_t>(tm) >> 2) & 3u)) & 3u));
    if (lane < h) {
      const float x = tm[lane];
      low16 |= __float_as_uint(x);
      tkey[lane] = fkey(x);
    }
    const int nv4 = (ntv - h) >> 2;
    const float4* tm4 = reinterpret_cast<const float4*>(tm + h);  // 16-byte aligned
    constexpr int kU = 8;
    for (int v0 = lane; v0 < nv4; v0 += 32 * kU) {
      float4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int vi = v0 + 32 * u;
        x[u] = vi < nv4 ? __ldg(tm4 + vi) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int vi = v0 + 32 * u;
        if (vi < nv4) {
          uint32_t* t4 = tkey + h + 4 * vi;
          low16 |= __float_as_uint(x[u].x) | __float_as_uint(x[u].y) | __float_as_uint(x[u].z) | __float_as_uint(x[u].w);
          t4[0] = fkey(x[u].x);
          t4[1] = fkey(x[u].y);
          t4[2] = fkey(x[u].z);
          t4[3] = fkey(x[u].w);
        }
      }
    }
    for (int i = h + 4 * nv4 + lane; i < ntv; i += 32) {
      const float x = tm[i];
      low16 |= __float_as_uint(x);
      tkey[i] = fkey(x);
    }
  }
  __syncwarp();
  // every tile maximum a bf16 value (the scan's are): the keys' low halves are then 0 (positive) or
  // 0xffff (negative) and carry no order, so the tiles can be picked on 32-bit words
  const bool tiles16 = __all_sync(0xffffffffu, (low16 & 0xffffu) == 0u) && ntv <= 0xffff;
  // (1) tiles: threshold + sort when it applies (on 32-bit words when the keys allow), else the radix select
  uint64_t srt[2], kth;
  uint32_t srt32[2], kth32;
  uint32_t* s_w32 = reinterpret_cast<uint32_t*>(s_w64[warp]);
  auto tword = [&](int i) -> uint64_t { return ((uint64_t)tkey[i] << 32) | (uint64_t)(0xffffffffu - (uint32_t)i); };
  auto tword32 = [&](int i) -> uint32_t { return (tkey[i] & 0xffff0000u) | (uint32_t)(0xffff - i); };
  if (tiles16 && warp_topk_sorted32(ntv, kt2, tword32, s_w32, srt32, kth32)) {
    int taken = 0;
    for (int i0 = 0; i0 < ntv; i0 += 32) {  // the kt2 tiles with word >= kth, in ascending tile order
      const int i = i0 + lane;
      const bool take = i < ntv && tword32(i) >= kth32;
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      if (take) tiles[taken + __popc(bt & ((1u << lane) - 1u))] = i;
      taken += __popc(bt);
    }
  } else if (warp_topk_sorted(ntv, kt2, tword, s_w64[warp], srt, kth)) {
    int taken = 0;
    for (int i0 = 0; i0 < ntv; i0 += 32) {  // the kt2 tiles with word >= kth, in ascending tile order
      const int i = i0 + lane;
      const bool take = i < ntv && tword(i) >= kth;
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      if (take) tiles[taken + __popc(bt & ((1u << lane) - 1u))] = i;
      taken += __popc(bt);
    }
  } else {
  uint32_t Tt;
  int above_t;
  warp_radix_select<32>(ntv, kt2, hist, [&](int i, bool& v, uint32_t& k) { v = true; k = tkey[i]; }, Tt, above_t);
  {
    int taken = 0, ties = 0;
    const int need_eq = kt2 - above_t;
    for (int i0 = 0; i0 < ntv; i0 += 32) {
      const int i = i0 + lane;
      const uint32_t k = i < ntv ? tkey[i] : 0u;
      const bool gt = i < ntv && k > Tt, eq = i < ntv && k == Tt;
      const unsigned beq = __ballot_sync(0xffffffffu, eq);
      const bool take = gt || (eq && ties + __popc(beq & ((1u << lane) - 1u)) < need_eq);
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      if (take) tiles[taken + __popc(bt & ((1u << lane) - 1u))] = i;
      taken += __popc(bt);
      ties += __popc(beq);
    }
  }
  }
  __syncwarp();
  // (2) candidate keys of the chosen tiles (ascending tile order) staged with 16-byte loads;
  //     positions >= n get key 0 (below every real key, which is >= 0x7f)
  const int m = kt2 * kMaxTile;
  for (int i0 = lane * 8; i0 < m; i0 += 32 * 8 * 4) {  // four 16-byte loads in flight per lane
    uint4 w[4];
    int pos[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + 32 * 8 * u;
      pos[u] = i < m ? tiles[i >> 5] * kMaxTile + (i & (kMaxTile - 1)) : 0;
      w[u] = i < m ? *reinterpret_cast<const uint4*>(srw + pos[u]) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + 32 * 8 * u;
      if (i < m) {
        const uint32_t wv[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t b = (wv[e >> 1] >> (16 * (e & 1))) & 0xffffu;
          ckey[i + e] = (pos[u] + e < n) ? (uint16_t)ukey16(b) : (uint16_t)0;
        }
      }
    }
  }
  __syncwarp();
  auto cand = [&](int i, bool& v, uint32_t& k) {
    k = ckey[i];
    v = k != 0u;
  };
  // candidate i is tile tiles[i >> 5], offset i & 31: ascending i is ascending position; 16-bit keys
  // and i < 4096, so (key << 16) | (0xffff - i) orders them as the reference does
  auto cword = [&](int i) -> uint32_t {
    const uint32_t k = ckey[i];
    return k ? (k << 16) | (uint32_t)(0xffff - i) : 0u;
  };
  int32_t* outp = a.sel + (int64_t)r * (a.ns + a.nl + a.k_top);
  if (warp_topk_sorted32(m, a.k_top, cword, s_w32, srt32, kth32)) {
    // the k winners, already in rank order (score desc, position asc)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      if (e < a.k_top) {
        const int i = 0xffff - (int)(srt32[h] & 0xffffu);
        s_pos[warp][e] = tiles[i >> 5] * kMaxTile + (i & (kMaxTile - 1));
      }
    }
    __syncwarp();
    for (int j = lane; j < a.k_top; j += 32) outp[a.ns + a.nl + j] = s_pos[warp][j];
  } else {
  uint32_t T;
  int above;
  warp_radix_select<16>(m, a.k_top, hist, cand, T, above);
  {
    int taken = 0, ties = 0;
    const int need_eq = a.k_top - above;
    for (int i0 = 0; i0 < m; i0 += 32) {
      const int i = i0 + lane;
      bool v = false;
      uint32_t k = 0u;
      if (i < m) cand(i, v, k);
      const bool gt = v && k > T, eq = v && k == T;
      const unsigned beq = __ballot_sync(0xffffffffu, eq);
      const bool take = gt || (eq && ties + __popc(beq & ((1u << lane) - 1u)) < need_eq);
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      const int slot = taken + __popc(bt & ((1u << lane) - 1u));
      if (take && slot < a.k_top) {
        s_pos[warp][slot] = tiles[i >> 5] * kMaxTile + (i & (kMaxTile - 1));
        s_key[warp][slot] = k;
      }
      taken += __popc(bt);
      ties += __popc(beq);
    }
    // (fewer candidates than k cannot happen for k_top <= n - ns - nl; pad with position 0)
    for (int j = taken + lane; j < a.k_top; j += 32) {
      s_pos[warp][j] = 0;
      s_key[warp][j] = 0u;
    }
  }
  __syncwarp();
  // (3) rank order (score desc, position asc)
  for (int j = lane; j < a.k_top; j += 32) {
    const uint32_t kj = s_key[warp][j];
    const int pj = s_pos[warp][j];
    int rank = 0;
    for (int i = 0; i < a.k_top; ++i) {
      const uint32_t ki = s_key[warp][i];
      const int pi = s_pos[warp][i];
      rank += (ki > kj || (ki == kj && pi < pj)) ? 1 : 0;
    }
    outp[a.ns + a.nl + rank] = pj;
  }
  }
  __syncwarp();
  for (int j = lane; j < a.k_top; j += 32) {
    const int t = s_pos[warp][j];
    if (t >= 0 && t < a.Lmax) srw[t] = 0xff80u;
  }
  for (int i = lane; i < a.ns + a.nl; i += 32) {
    const int t = i < a.ns ? i : n - a.nl + (i - a.ns);
    outp[i] = t;
    if (t >= 0 && t < a.Lmax) srw[t] = 0xff80u;
  }
}

// ------------------------------------------------------------------------ token append (runner helper)
// One CTA: the new token's K and V rows of every (request, KV head) are written at position
// n + offset (n = n_dev[0] as read at the start); then, with `advance`, n_dev[0] = n + 1 and
// kv_idx[0] = n.  A single CTA so that every row is written before the counters change.
constexpr int kApThreads = 1024;
__global__ void __launch_bounds__(kApThreads) append_kv_kernel(__nv_bfloat16* K, __nv_bfloat16* V, int rows, int Lmax,
                                                             const __nv_bfloat16* k_new, const __nv_bfloat16* v_new,
                                                             int32_t* n_dev, int offset, int advance, int64_t* kv_idx) {
  const int n = *n_dev;
  const int p = n + offset;
  if (p >= 0 && p < Lmax) {
    const int vec = rows * kD / 8;  // 16-byte vectors per tensor
    constexpr int kU = 8;           // loads a thread issues before its stores
    for (int i0 = threadIdx.x; i0 < 2 * vec; i0 += kApThreads * kU) {
      uint4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = i0 + kApThreads * u;
        const int t = i < vec ? 0 : 1, j = i - t * vec;
        x[u] = i < 2 * vec ? reinterpret_cast<const uint4*>(t ? v_new : k_new)[j] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = i0 + kApThreads * u;
        if (i < 2 * vec) {
          const int t = i < vec ? 0 : 1, j = i - t * vec;
          const int row = j / (kD / 8), part = j - row * (kD / 8);
          reinterpret_cast<uint4*>((t ? V : K) + ((int64_t)row * Lmax + p) * kD)[part] = x[u];
        }
      }
    }
  }
  __syncthreads();
  if (advance && threadIdx.x == 0) {
    *n_dev = n + 1;
    if (kv_idx != nullptr) *kv_idx = n;
  }
}

}  // namespace
}  // namespace oa

// ------------------------------------------------------------------------ C ABI
using namespace oa;

namespace {
int index_update_entry(const char* fn, void* K, void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C, int8_t* codes,
                       const float* U, const float* scale, const void* W, const float* colmean, const float* cent,
                       int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv, int32_t* reclist, int32_t* reccnt,
                       int rmax, const void* q, int64_t q_stride, void* zq, const int32_t* n_dev, const void* k_new,
                       const void* v_new, void* stream) {
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= 4096, "%s: bad sizes B=%lld Lmax=%lld C=%lld", fn, (long long)B,
             (long long)Lmax, (long long)C);
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(Lmax < (1ll << 31) / 1, "%s: Lmax too large", fn);
  OA_REQUIRE(K && V && codes && U && scale && W && colmean && cent && asg && nb && Sk && Sk2 && Sv && n_dev,
             "%s: null pointer", fn);
  OA_REQUIRE(q == nullptr || zq != nullptr, "%s: q given without zq", fn);
  OA_REQUIRE(reclist == nullptr || (reccnt != nullptr && rmax > 0), "%s: reclist needs reccnt and rmax > 0", fn);
  OA_REQUIRE((k_new == nullptr) == (v_new == nullptr), "%s: k_new and v_new are given together", fn);
  IndexArgs a{static_cast<const __nv_bfloat16*>(K), static_cast<const __nv_bfloat16*>(V), codes, U, scale,
              static_cast<const __nv_bfloat16*>(W), colmean, cent, asg, nb, Sk, Sk2, Sv, reclist, reccnt, rmax,
              static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<__nv_bfloat16*>(zq), n_dev,
              (int)Lmax, (int)C, static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new)};
  const size_t smem = (size_t)std::min<int64_t>(C, kIuCentCache) * kRC * sizeof(float);
  OA_REQUIRE(oa_aligned16(cent) && oa_aligned16(U) && oa_aligned16(W), "%s: U / W / cent must be 16-byte aligned", fn);
  if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(index_update_kernel), smem, fn, true)) return rc;
  index_update_kernel<<<(unsigned)(B * kG * hkv), 128, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}
}  // namespace

extern "C" int oa_index_update(const void* K, const void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C,
                               int8_t* codes,
                               const float* U, const float* scale, const void* W, const float* colmean,
                               const float* cent, int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv,
                               int32_t* reclist, int32_t* reccnt, int rmax, const void* q, int64_t q_stride,
                               void* zq, const int32_t* n_dev, void* stream) {
  return index_update_entry("oa_index_update", const_cast<void*>(K), const_cast<void*>(V), B, hkv, Lmax, C, codes, U,
                            scale, W, colmean, cent, asg, nb, Sk, Sk2, Sv, reclist, reccnt, rmax, q, q_stride, zq,
                            n_dev, nullptr, nullptr, stream);
}

extern "C" int oa_index_update_append(void* K, void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C,
                                      const void* k_new,
                                      const void* v_new, int8_t* codes, const float* U, const float* scale,
                                      const void* W, const float* colmean, const float* cent, int32_t* asg, float* nb,
                                      float* Sk, float* Sk2, float* Sv, int32_t* reclist, int32_t* reccnt, int rmax,
                                      const void* q, int64_t q_stride, void* zq, const int32_t* n_dev,
                                      void* stream) {
  const char* fn = "oa_index_update_append";
  OA_REQUIRE(k_new && v_new, "%s: null k_new / v_new", fn);
  return index_update_entry(fn, K, V, B, hkv, Lmax, C, codes, U, scale, W, colmean, cent, asg, nb, Sk, Sk2, Sv, reclist,
                            reccnt, rmax, q, q_stride, zq, n_dev, k_new, v_new, stream);
}

extern "C" int oa_append_kv(void* K, void* V, int64_t B, int64_t hkv, int64_t Lmax, const void* k_new,
                            const void* v_new, int32_t* n_dev, int offset, int advance, int64_t* kv_idx, void* stream) {
  const char* fn = "oa_append_kv";
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(B > 0 && Lmax > 0 && Lmax < (1ll << 31) && B * kHKV * kD / 8 * 2 < (1ll << 31), "%s: bad sizes", fn);
  OA_REQUIRE(K && V && k_new && v_new && n_dev, "%s: null pointer", fn);
  OA_REQUIRE(oa_aligned16(K) && oa_aligned16(V) && oa_aligned16(k_new) && oa_aligned16(v_new),
             "%s: K, V, k_new and v_new must be 16-byte aligned", fn);
  append_kv_kernel<<<1, kApThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(K), static_cast<__nv_bfloat16*>(V), (int)(B * hkv), (int)Lmax,
      static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new), n_dev, offset,
      advance ? 1 : 0, kv_idx);
  return oa_check_launch(fn);
}

extern "C" int oa_qgs_scan(const int8_t* codes, const void* zq, int64_t B, int64_t hkv, int64_t Lmax,
                           const int32_t* n_dev, int ns, int nl, void* scores, int64_t score_stride, float* tile_max,
                           int64_t tile_max_stride, int32_t* status, void* stream) {
  const char* fn = "oa_qgs_scan";
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(B > 0 && Lmax > 0 && Lmax < (1ll << 30), "%s: bad sizes", fn);
  OA_REQUIRE(codes && zq && n_dev && scores && tile_max, "%s: null pointer", fn);
  OA_REQUIRE(oa_aligned16(codes), "%s: codes must be 16-byte aligned", fn);
  const int NT = (int)((Lmax + kMaxTile - 1) / kMaxTile);
  OA_REQUIRE(score_stride >= Lmax && tile_max_stride >= NT, "%s: score stride %lld < Lmax or tile-max stride < %d",
             fn, (long long)score_stride, NT);
  OA_REQUIRE(score_stride % 8 == 0 && oa_aligned16(scores), "%s: score rows must be 16-byte aligned", fn);
  OA_REQUIRE(ns >= 0 && nl >= 0, "%s: negative sink/local", fn);
  ScanArgs a{codes, static_cast<const __nv_bfloat16*>(zq), n_dev, ns, nl, (int)Lmax, NT,
             static_cast<uint16_t*>(scores), score_stride, tile_max, tile_max_stride, status};
  const int nsteps = (int)((Lmax + kTile - 1) / kTile);
  dim3 grid((unsigned)(B * hkv), (unsigned)((nsteps + kTilesPerCta - 1) / kTilesPerCta));
  qgs_scan_kernel<<<grid, kScanThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_qgs_select(void* scores, int64_t score_stride, const float* tile_max, int64_t tile_max_stride,
                             int64_t R, int64_t Lmax, const int32_t* n_dev, int ns, int nl, int k_top, int32_t* sel,
                             void* stream) {
  const char* fn = "oa_qgs_select";
  OA_REQUIRE(R > 0 && R < (1ll << 31) && Lmax > 0 && Lmax < (1ll << 30), "%s: bad sizes", fn);
  OA_REQUIRE(scores && tile_max && n_dev && sel, "%s: null pointer", fn);
  OA_REQUIRE(k_top >= 1 && 2 * k_top <= kMaxKT2, "%s: k_top=%d outside [1, %d]", fn, k_top, kMaxKT2 / 2);
  OA_REQUIRE(ns >= 0 && nl >= 0, "%s: negative sink/local", fn);
  const int NT = (int)((Lmax + kMaxTile - 1) / kMaxTile);
  OA_REQUIRE(score_stride % 8 == 0 && oa_aligned16(scores), "%s: scores rows must be 16-byte aligned", fn);
  const int NT_pad = (NT + 3) & ~3;
  const int kt2_max = std::min(2 * k_top, NT);
  SelectArgs a{static_cast<uint16_t*>(scores), score_stride, tile_max, tile_max_stride, n_dev, (int)R, ns, nl, k_top,
               NT, (int)Lmax, sel, NT_pad, kt2_max};
  const size_t smem = (size_t)kSelWarps * (NT_pad * 4 + (size_t)kt2_max * kMaxTile * 2);
  OA_REQUIRE(smem <= 200 * 1024, "%s: Lmax=%lld and k_top=%d need too much shared memory", fn, (long long)Lmax, k_top);
  if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(qgs_select_kernel), smem, fn)) return rc;
  qgs_select_kernel<<<(unsigned)((R + kSelWarps - 1) / kSelWarps), kSelWarps * 32, smem,
                      static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}
