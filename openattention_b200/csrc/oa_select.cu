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
};

__global__ void __launch_bounds__(128) index_update_kernel(const IndexArgs a) {
  const int kv = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = __ldg(a.n_dev) - 1;
  __shared__ float kf[kD], vf[kD], qf[kG][kD], zp[kG][kRC];
  const bool have_tok = pos >= 0 && pos < a.Lmax;
  if (have_tok) {
    kf[tid] = __bfloat162float(a.K[((int64_t)kv * a.Lmax + pos) * kD + tid]);
    vf[tid] = __bfloat162float(a.V[((int64_t)kv * a.Lmax + pos) * kD + tid]);
  }
  if (a.q != nullptr) {
#pragma unroll
    for (int g = 0; g < kG; ++g) qf[g][tid] = __bfloat162float(a.q[(int64_t)(kv * kG + g) * a.q_stride + tid]);
  }
  __syncthreads();
  const float* Uk = a.U + (int64_t)kv * kD * kRQ;
  // query projection zq[r, j] = bf16((q . U[:, j]) * scale_j), d ascending
  if (a.q != nullptr) {
    const int g = tid >> 5, j = tid & 31;
    float acc = 0.f;
    for (int d = 0; d < kD; ++d) acc = __fmaf_rn(qf[g][d], __ldg(&Uk[d * kRQ + j]), acc);
    a.zq[(int64_t)(kv * kG + g) * kRQ + j] = __float2bfloat16_rn(__fmul_rn(acc, __ldg(&a.scale[kv * kRQ + j])));
  }
  if (!have_tok) return;
  // QGS code of the new key (per KV head)
  if (tid < kRQ) {
    const int j = tid;
    float acc = 0.f;
    for (int d = 0; d < kD; ++d) acc = __fmaf_rn(kf[d], __ldg(&Uk[d * kRQ + j]), acc);
    float c = rintf(__fdiv_rn(acc, __ldg(&a.scale[kv * kRQ + j])));
    c = fminf(fmaxf(c, -127.f), 127.f);
    a.codes[((int64_t)kv * a.Lmax + pos) * kRQ + j] = (int8_t)c;
  }
  // rank-16 QGC projection per query head: zp = bf16(k . W) - colmean
  if (tid < kG * kRC) {
    const int g = tid >> 4, c = tid & 15;
    const int r = kv * kG + g;
    const __nv_bfloat16* Wr = a.W + (int64_t)r * kD * kRC;
    float acc = 0.f;
    for (int d = 0; d < kD; ++d) acc = __fmaf_rn(kf[d], __bfloat162float(Wr[d * kRC + c]), acc);
    zp[g][c] = __fsub_rn(bf_round(acc), __ldg(&a.colmean[r * kRC + c]));
  }
  __syncthreads();
  // nearest centroid (warp g <-> query head g); ties -> lower cluster id
  const int g = warp;
  const int r = kv * kG + g;
  const float* ce = a.cent + (int64_t)r * a.C * kRC;
  float bestv = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = lane; i < a.C; i += 32) {
    float dot = 0.f, nrm = 0.f;
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      const float x = __ldg(&ce[i * kRC + c]);
      dot = __fmaf_rn(zp[g][c], x, dot);
      nrm = __fmaf_rn(x, x, nrm);
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
  const int cid = besti == 0x7fffffff ? 0 : besti;
  float* sk = a.Sk + ((int64_t)r * a.C + cid) * kD;
  float* sk2 = a.Sk2 + ((int64_t)r * a.C + cid) * kD;
  float* sv = a.Sv + ((int64_t)r * a.C + cid) * kD;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    sk[d] = __fadd_rn(sk[d], kf[d]);
    sk2[d] = __fadd_rn(sk2[d], __fmul_rn(kf[d], kf[d]));
    sv[d] = __fadd_rn(sv[d], vf[d]);
  }
  if (lane == 0) {
    a.asg[(int64_t)r * a.Lmax + pos] = cid;
    a.nb[(int64_t)r * a.C + cid] = __fadd_rn(a.nb[(int64_t)r * a.C + cid], 1.f);
    if (a.reclist != nullptr) {
      const int cnt = a.reccnt[(int64_t)r * a.C + cid];
      if (cnt < a.rmax) a.reclist[((int64_t)r * a.C + cid) * a.rmax + cnt] = pos;
      a.reccnt[(int64_t)r * a.C + cid] = cnt + 1;
    }
  }
}

// ------------------------------------------------------------------------ QGS scan (int8 MMA)
constexpr int kTile = 256;         // tokens per tile maximum
constexpr int kScanThreads = 256;  // 8 warps x 32 tokens = one tile per step
constexpr int kTilesPerCta = 4;

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

__global__ void __launch_bounds__(kScanThreads) qgs_scan_kernel(const ScanArgs a) {
  const int kv = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int n = __ldg(a.n_dev);
  __shared__ int8_t limb[kG][4][kRQ];  // [head][limb][j]
  __shared__ int sS[kG];
  __shared__ float s_max[8][kG];
  // fixed-point image of each head's zq (one warp per head)
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
  // B fragments: column n = gid -> head 2m + gid/4, limb gid%4; rows k = tig*4..+3 and 16 + tig*4..+3
  uint32_t bf[2][2];
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int h = 2 * m + (gid >> 2), k = gid & 3;
    bf[m][0] = *reinterpret_cast<const uint32_t*>(&limb[h][k][tig * 4]);
    bf[m][1] = *reinterpret_cast<const uint32_t*>(&limb[h][k][16 + tig * 4]);
  }
  const int fin_head[2] = {0 + (tig >> 1), 2 + (tig >> 1)};
  const int S_h[2] = {sS[fin_head[0]], sS[fin_head[1]]};
  const int8_t* cbase = a.codes + (int64_t)kv * a.Lmax * kRQ;
  const int t_begin = blockIdx.y * kTilesPerCta;
  for (int tile = t_begin; tile < t_begin + kTilesPerCta && tile < a.NT; ++tile) {
    const int t0 = tile * kTile;
    float hmax[2] = {-INFINITY, -INFINITY};  // for heads fin_head[0], fin_head[1]
    if (t0 < n) {
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int tb = t0 + warp * 32 + grp * 16;
        const int ta = tb + gid, tb8 = tb + gid + 8;
        uint32_t af[4];
        const uint32_t* p0 = reinterpret_cast<const uint32_t*>(cbase + (int64_t)ta * kRQ);
        const uint32_t* p1 = reinterpret_cast<const uint32_t*>(cbase + (int64_t)tb8 * kRQ);
        const bool ok0 = ta < a.Lmax, ok1 = tb8 < a.Lmax;
        af[0] = ok0 ? __ldg(p0 + tig) : 0u;
        af[1] = ok1 ? __ldg(p1 + tig) : 0u;
        af[2] = ok0 ? __ldg(p0 + 4 + tig) : 0u;
        af[3] = ok1 ? __ldg(p1 + 4 + tig) : 0u;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          int d[4];
          mma_s8(d, af, bf[m][0], bf[m][1]);
          // exchange limb pairs with the partner lane (tig ^ 1) holding the other two limbs
          int e[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) e[i] = __shfl_xor_sync(0xffffffffu, d[i], 1);
          // limbs 0,1 live on even tig, limbs 2,3 on odd tig
          const int* lo = (tig & 1) ? e : d;
          const int* hi = (tig & 1) ? d : e;
          const int row = tig & 1;  // even tig finalises token gid, odd tig token gid+8
          const long long tot = (long long)lo[2 * row] + ((long long)lo[2 * row + 1] << 8) +
                                ((long long)hi[2 * row] << 16) + ((long long)hi[2 * row + 1] << 24);
          const int t = row ? tb8 : ta;
          float f = scale_pow2(__ll2float_rn(tot), -S_h[m]);
          uint16_t sb = f2bf_bits(f);
          if (t < a.ns || t >= n - a.nl || t >= n) sb = 0xff80u;
          if (t < a.Lmax) {
            a.scores[(int64_t)(kv * kG + fin_head[m]) * a.sw + t] = sb;
            hmax[m] = fmaxf(hmax[m], __uint_as_float((uint32_t)sb << 16));
          }
        }
      }
    }
    // tile maximum per head: lanes with tig>>1 == h hold head 2m + h
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      float v = hmax[m];
      // reduce over lanes sharing (tig >> 1): xor over gid bits (4, 8, 16) and tig bit 0 (1)
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
      if (lane == 0) s_max[warp][2 * m] = v;      // tig 0 -> head 2m
      if (lane == 2) s_max[warp][2 * m + 1] = v;  // tig 2 -> head 2m + 1
    }
    __syncthreads();
    if (tid < kG) {
      float v = -INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) v = fmaxf(v, s_max[w][tid]);
      a.tmax[(int64_t)(kv * kG + tid) * a.tm_stride + tile] = v;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------ exact row top-k
struct SelectArgs {
  uint16_t* scores;
  int64_t sw;
  const float* tmax;
  int64_t tm_stride;
  const int32_t* n_dev;
  int ns, nl, k_top, NT, Lmax;
  int kt2_max;
  int32_t* sel;
};

__device__ __forceinline__ uint32_t fkey(float x) {  // ascending float -> ascending uint32
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint32_t ukey16(uint32_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, off);
    v = o > v ? o : v;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) v = red[w] > v ? red[w] : v;
  return v;
}

__global__ void __launch_bounds__(256) qgs_select_kernel(const SelectArgs a) {
  extern __shared__ unsigned char smem_raw[];
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const int n = __ldg(a.n_dev);
  const int ntv = min(a.NT, (n + kTile - 1) / kTile);
  const int kt2 = min(2 * a.k_top, ntv);
  // tile keys: (max, lowest tile first) -> pick kt2 largest by repeated block argmax over a small list
  unsigned long long* red = reinterpret_cast<unsigned long long*>(smem_raw);          // 8
  int* chosen = reinterpret_cast<int*>(smem_raw + 64);                                  // kt2_max
  uint16_t* cand = reinterpret_cast<uint16_t*>(smem_raw + 64 + 4 * a.kt2_max);         // kt2_max * 256
  unsigned char* taken = reinterpret_cast<unsigned char*>(cand + (size_t)a.kt2_max * kTile);  // kt2_max*256
  const float* tm = a.tmax + (int64_t)r * a.tm_stride;
  const uint16_t* sr = a.scores + (int64_t)r * a.sw;
  // per-thread strided tile keys; kt2 rounds of block argmax (NT <= a few thousand)
  for (int round = 0; round < kt2; ++round) {
    unsigned long long best = 0ull;
    for (int t = tid; t < ntv; t += blockDim.x) {
      bool used = false;
      for (int i = 0; i < round; ++i) used |= (chosen[i] == t);
      if (used) continue;
      const unsigned long long key = ((unsigned long long)fkey(tm[t]) << 32) | (0xffffffffu - (uint32_t)t);
      best = key > best ? key : best;
    }
    best = block_max_u64(best, red);
    if (tid == 0) chosen[round] = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
    __syncthreads();
  }
  // candidate scores of the chosen tiles
  const int ncand = kt2 * kTile;
  for (int i = tid; i < ncand; i += blockDim.x) {
    const int t = chosen[i / kTile] * kTile + (i % kTile);
    const bool ok = t < n;
    cand[i] = ok ? (uint16_t)ukey16(sr[t]) : (uint16_t)0;
    taken[i] = ok ? 0 : 1;
  }
  __syncthreads();
  int32_t* out = a.sel + (int64_t)r * (a.ns + a.nl + a.k_top);
  for (int k = 0; k < a.k_top; ++k) {
    unsigned long long best = 0ull;
    for (int i = tid; i < ncand; i += blockDim.x) {
      if (taken[i]) continue;
      const uint32_t t = (uint32_t)(chosen[i / kTile] * kTile + (i % kTile));
      const unsigned long long key = ((unsigned long long)(cand[i] + 1u) << 32) | (0xffffffffu - t);
      best = key > best ? key : best;
    }
    best = block_max_u64(best, red);
    const int t = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
    if (best == 0ull) {
      if (tid == 0) out[a.ns + a.nl + k] = 0;  // fewer candidates than k_top (cannot happen for k_top <= n)
    } else {
      if (tid == 0) out[a.ns + a.nl + k] = t;
      for (int i = tid; i < ncand; i += blockDim.x)
        if (chosen[i / kTile] * kTile + (i % kTile) == t) taken[i] = 1;
    }
    __syncthreads();
  }
  // sink, local; selected scores -> -inf (they go last in their cluster for the within-cluster top-q)
  uint16_t* srw = a.scores + (int64_t)r * a.sw;
  for (int i = tid; i < a.ns + a.nl; i += blockDim.x) {
    const int t = i < a.ns ? i : n - a.nl + (i - a.ns);
    out[i] = t;
    if (t >= 0 && t < a.Lmax) srw[t] = 0xff80u;
  }
  __syncthreads();
  for (int k = tid; k < a.k_top; k += blockDim.x) {
    const int t = out[a.ns + a.nl + k];
    if (t >= 0 && t < a.Lmax) srw[t] = 0xff80u;
  }
}

}  // namespace
}  // namespace oa

// ------------------------------------------------------------------------ C ABI
using namespace oa;

extern "C" int oa_index_update(const void* K, const void* V, int64_t B, int64_t Lmax, int64_t C, int8_t* codes,
                               const float* U, const float* scale, const void* W, const float* colmean,
                               const float* cent, int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv,
                               int32_t* reclist, int32_t* reccnt, int rmax, const void* q, int64_t q_stride,
                               void* zq, const int32_t* n_dev, void* stream) {
  const char* fn = "oa_index_update";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= 4096, "%s: bad sizes B=%lld Lmax=%lld C=%lld", fn, (long long)B,
             (long long)Lmax, (long long)C);
  OA_REQUIRE(Lmax < (1ll << 31) / 1, "%s: Lmax too large", fn);
  OA_REQUIRE(K && V && codes && U && scale && W && colmean && cent && asg && nb && Sk && Sk2 && Sv && n_dev,
             "%s: null pointer", fn);
  OA_REQUIRE(q == nullptr || zq != nullptr, "%s: q given without zq", fn);
  OA_REQUIRE(reclist == nullptr || (reccnt != nullptr && rmax > 0), "%s: reclist needs reccnt and rmax > 0", fn);
  IndexArgs a{static_cast<const __nv_bfloat16*>(K), static_cast<const __nv_bfloat16*>(V), codes, U, scale,
              static_cast<const __nv_bfloat16*>(W), colmean, cent, asg, nb, Sk, Sk2, Sv, reclist, reccnt, rmax,
              static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<__nv_bfloat16*>(zq), n_dev,
              (int)Lmax, (int)C};
  index_update_kernel<<<(unsigned)(B * kHKV), 128, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_qgs_scan(const int8_t* codes, const void* zq, int64_t B, int64_t Lmax, const int32_t* n_dev, int ns,
                           int nl, void* scores, int64_t score_stride, float* tile_max, int64_t tile_max_stride,
                           void* stream) {
  const char* fn = "oa_qgs_scan";
  OA_REQUIRE(B > 0 && Lmax > 0 && Lmax < (1ll << 30), "%s: bad sizes", fn);
  OA_REQUIRE(codes && zq && n_dev && scores && tile_max, "%s: null pointer", fn);
  OA_REQUIRE(oa_aligned16(codes), "%s: codes must be 16-byte aligned", fn);
  const int NT = (int)((Lmax + kTile - 1) / kTile);
  OA_REQUIRE(score_stride >= Lmax && tile_max_stride >= NT, "%s: score stride %lld < Lmax or tile-max stride < %d",
             fn, (long long)score_stride, NT);
  OA_REQUIRE(ns >= 0 && nl >= 0, "%s: negative sink/local", fn);
  ScanArgs a{codes, static_cast<const __nv_bfloat16*>(zq), n_dev, ns, nl, (int)Lmax, NT,
             static_cast<uint16_t*>(scores), score_stride, tile_max, tile_max_stride};
  dim3 grid((unsigned)(B * kHKV), (unsigned)((NT + kTilesPerCta - 1) / kTilesPerCta));
  qgs_scan_kernel<<<grid, kScanThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_qgs_select(void* scores, int64_t score_stride, const float* tile_max, int64_t tile_max_stride,
                             int64_t R, int64_t Lmax, const int32_t* n_dev, int ns, int nl, int k_top, int32_t* sel,
                             void* stream) {
  const char* fn = "oa_qgs_select";
  OA_REQUIRE(R > 0 && Lmax > 0 && Lmax < (1ll << 30), "%s: bad sizes", fn);
  OA_REQUIRE(scores && tile_max && n_dev && sel, "%s: null pointer", fn);
  OA_REQUIRE(k_top >= 1 && k_top <= 64, "%s: k_top=%d outside [1, 64]", fn, k_top);
  OA_REQUIRE(ns >= 0 && nl >= 0, "%s: negative sink/local", fn);
  const int NT = (int)((Lmax + kTile - 1) / kTile);
  const int kt2_max = std::min(2 * k_top, NT);
  SelectArgs a{static_cast<uint16_t*>(scores), score_stride, tile_max, tile_max_stride, n_dev, ns, nl, k_top, NT,
               (int)Lmax, kt2_max, sel};
  const size_t smem = 64 + 4 * (size_t)kt2_max + (size_t)kt2_max * kTile * 3 + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(qgs_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
  }
  qgs_select_kernel<<<(unsigned)R, 256, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}
