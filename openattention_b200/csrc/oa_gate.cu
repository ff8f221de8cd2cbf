// Per-step selection back half on sm_100a: ErrorGate + hierarchical water-filling, within-cluster
// top-q, and the residual proxies (one CTA per query-head row in each kernel).
//
// ErrorGate restates _k_errorgate (inference/ours_fused.py:122-154; eager methods_eager.py:613-627),
// water-filling _k_waterfill / Ours.hier_quota (inference/ours_fused.py:158-216,
// methods_eager.py:558-581), top-q _k_topq_d2 (inference/ours_graph.py:93-166) and the residual
// _k_resid_scatter + _k_resid_norm (inference/ours_fused.py:367-407) without atomics.
//
// Every floating-point value that decides an index (ErrorGate score, weights, lambda, quotas) is
// computed by a fixed operation sequence: 128-term dots in the warp-tree order (lane l sums
// d = l, l+32, l+64, l+96 by fma, then an xor butterfly 16..1), the own double-precision ln / exp /
// erf of oa_math.cuh, sorts with explicit (value, cluster) tie-breaks, and the weight suffix sums
// accumulated in double from the end.
#include "oa_common.cuh"
#include "oa_math.cuh"
#include "oa_warp.cuh"

#include <cooperative_groups.h>
#include "../../include/openattention_b200.h"

namespace oa {
namespace {

constexpr int kMaxC = 256;
constexpr int kGateThreads = 256;

// A quota as the whole number of tokens it allots, clamped to [0, E].  The water-filling's quotas are
// whole numbers in that range already; a value a caller passes outside it (negative, NaN, above E)
// then cannot carry a prefix of quotas outside the expanded list.
__device__ __forceinline__ int quota_int(float x, int E) { return x > 0.f ? (int)fminf(x, (float)E) : 0; }

__device__ __forceinline__ float warp_tree_dot(const float (&a)[4], const float (&b)[4]) {
  float v = __fmul_rn(a[0], b[0]);
  v = __fmaf_rn(a[1], b[1], v);
  v = __fmaf_rn(a[2], b[2], v);
  v = __fmaf_rn(a[3], b[3], v);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// ------------------------------------------------------------------------ ErrorGate + water-filling
// ascending float -> ascending uint32, both zeros mapped to the key of +0 (they compare equal)
__device__ __forceinline__ uint32_t fkey_eg(float x) {
  const uint32_t b = __float_as_uint(x == 0.f ? 0.f : x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct GateArgs {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const __nv_bfloat16* K;
  int Lmax, C, NS;
  const int32_t* asg;
  const int32_t* sel;
  const float* Sk;
  const float* Sk2;
  const float* nb;
  float E;
  float* score;
  float* nt;
  float* quota;
  float* zdot;  // may be null
  int32_t* status;
};


// One CTA of 2 warps per row, so that every row of a batch is resident at once (the work of a row is
// a chain of short dependent steps; rows in parallel hide its latency).  Warp w owns the clusters
// w + 2k and streams their Sk / Sk2 rows (lane l holds dims 4l .. 4l+3, one 16-byte load) in batches of four,
// the next batch in flight while one is used; the selected tokens' K rows are staged in shared
// memory and subtracted, in list order, from their clusters; the two dots per cluster use the fixed
// warp-tree order.  The scalar tail (ln, erf, ln) and the water-filling run one thread per cluster
// (threads c, c + 64, ...): ranks by counting, the integer prefix of the caps in ratio order (one
// warp) beside the double suffix sum of the weights (one thread of the other warp).
constexpr int kEgThreads = 64;
constexpr int kEgB = 4;            // clusters per batch per warp
constexpr int kEgSelCache = 64;    // selected tokens whose K rows are staged in shared memory

struct EgShared {
  float *score, *nt, *lg, *zd, *sd, *w, *cap, *ratio, *qb, *capo, *wo, *rato, *cex, *wsuf, *inv;
  int *ord, *rank2, *ord2, *nsel, *selc, *selt;
  __nv_bfloat16* selk;
};

size_t eg_smem_bytes(int C, int NS) {
  const size_t c4 = (size_t)((C + 3) & ~3);
  const size_t ns4 = (size_t)((NS + 3) & ~3);
  return c4 * 4 * 19 + ns4 * 4 * 2 + (size_t)std::min(NS, kEgSelCache) * kD * 2;  // 15 fp32 + 4 int per cluster
}

template <int NT>
__global__ void __launch_bounds__(NT, NT == 64 ? 8 : 2) errorgate_waterfill_kernel(const GateArgs a) {
  constexpr int kW = NT / 32;  // warps
  extern __shared__ __align__(16) unsigned char eg_smem[];
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kv = r / kG;
  const int C = a.C, NS = a.NS;
  __shared__ float s_red[kW];
  __shared__ int s_redi[kW];
  EgShared S;
  {
    unsigned char* p = eg_smem;
    const int c4 = (C + 3) & ~3, ns4 = (NS + 3) & ~3;
    float* f = reinterpret_cast<float*>(p);
    S.score = f;
    S.nt = f + c4;
    S.lg = f + 2 * c4;
    S.zd = f + 3 * c4;
    S.sd = f + 4 * c4;
    S.w = f + 5 * c4;
    S.cap = f + 6 * c4;
    S.ratio = f + 7 * c4;
    S.qb = f + 8 * c4;
    S.capo = f + 9 * c4;
    S.wo = f + 10 * c4;
    S.rato = f + 11 * c4;
    S.cex = f + 12 * c4;
    S.wsuf = f + 13 * c4;
    S.inv = f + 14 * c4;
    p += sizeof(float) * 15 * c4;
    S.ord = reinterpret_cast<int*>(p);
    p += sizeof(int) * c4;
    S.rank2 = reinterpret_cast<int*>(p);
    p += sizeof(int) * c4;
    S.ord2 = reinterpret_cast<int*>(p);
    p += sizeof(int) * c4;
    S.nsel = reinterpret_cast<int*>(p);
    p += sizeof(int) * c4;
    S.selc = reinterpret_cast<int*>(p);
    p += sizeof(int) * ns4;
    S.selt = reinterpret_cast<int*>(p);
    p += sizeof(int) * ns4;
    S.selk = reinterpret_cast<__nv_bfloat16*>(p);
  }
  const int64_t rC = (int64_t)r * C;
  const __nv_bfloat16* Kr = a.K + (int64_t)kv * a.Lmax * kD;
  // ---- the first two batches of pooled-sum rows go out first: they depend on nothing
  float ck[kEgB][4], ck2[kEgB][4], nk[kEgB][4], nk2[kEgB][4];  // this batch, the next one
  auto fetch = [&](int b, float (&x)[kEgB][4], float (&x2)[kEgB][4]) {
#pragma unroll
    for (int k = 0; k < kEgB; ++k) {
      const int c = warp + kW * (b * kEgB + k);
      const int64_t base = (rC + min(c, C - 1)) * kD;
      const float4 u = c < C ? __ldg(reinterpret_cast<const float4*>(a.Sk + base) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 u2 = c < C ? __ldg(reinterpret_cast<const float4*>(a.Sk2 + base) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
      x[k][0] = u.x; x[k][1] = u.y; x[k][2] = u.z; x[k][3] = u.w;
      x2[k][0] = u2.x; x2[k][1] = u2.y; x2[k][2] = u2.z; x2[k][3] = u2.w;
    }
  };
  const int nbatch = (C + kW * kEgB - 1) / (kW * kEgB);
  fetch(0, ck, ck2);
  if (nbatch > 1) fetch(1, nk, nk2);
  // ---- selected tokens: their clusters and their K rows are fetched side by side
  for (int j = tid; j < NS; j += NT) {
    const int t = a.sel[(int64_t)r * NS + j];
    const bool v = t >= 0 && t < a.Lmax;
    S.selt[j] = v ? t : -1;
    S.selc[j] = v ? a.asg[(int64_t)r * a.Lmax + t] : -1;
  }
  {  // K rows of the selected tokens: a thread's indices first, then all its row loads, then the stores
    constexpr int kSU = 4;
    const int ne = min(NS, kEgSelCache) * 16;
    for (int e0 = tid; e0 < ne; e0 += NT * kSU) {
      int t[kSU];
#pragma unroll
      for (int u = 0; u < kSU; ++u) {
        const int e = e0 + NT * u;
        t[u] = e < ne ? a.sel[(int64_t)r * NS + (e >> 4)] : -1;
      }
      uint4 x[kSU];
#pragma unroll
      for (int u = 0; u < kSU; ++u) {
        const int e = e0 + NT * u;
        x[u] = (t[u] >= 0 && t[u] < a.Lmax) ? __ldg(reinterpret_cast<const uint4*>(Kr + (int64_t)t[u] * kD + (e & 15) * 8))
                                            : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kSU; ++u) {
        const int e = e0 + NT * u;
        if (t[u] >= 0 && t[u] < a.Lmax) *reinterpret_cast<uint4*>(S.selk + (e >> 4) * kD + (e & 15) * 8) = x[u];
      }
    }
  }
  __syncthreads();
  float qv[4], q2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qv[i] = __bfloat162float(a.q[(int64_t)r * a.q_stride + 4 * lane + i]);
    q2[i] = __fmul_rn(qv[i], qv[i]);
  }
  // tail counts and ln n_t, one thread per cluster, while the rows are in flight
  for (int c = tid; c < C; c += NT) {
    float ntc = a.nb[rC + c];
    int ns_c = 0;
    for (int j = 0; j < NS; ++j)
      if (S.selc[j] == c) {
        ntc = __fsub_rn(ntc, 1.f);
        ++ns_c;
      }
    S.nt[c] = ntc;
    S.nsel[c] = ns_c;
    S.inv[c] = __fdiv_rn(1.f, fmaxf(ntc, 1.f));
    S.lg[c] = ln_f(fmaxf(ntc, 1.f));
  }
  __syncthreads();
  // ---- ErrorGate dots, batch by batch
  for (int b = 0; b < nbatch; ++b) {
    float sk[kEgB][4], sk2[kEgB][4];
#pragma unroll
    for (int k = 0; k < kEgB; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sk[k][i] = ck[k][i];
        sk2[k][i] = ck2[k][i];
        ck[k][i] = nk[k][i];
        ck2[k][i] = nk2[k][i];
      }
    if (b + 2 < nbatch) fetch(b + 2, nk, nk2);
    const int cb = warp + kW * b * kEgB;  // clusters cb + kW * k
    int any = 0;
#pragma unroll
    for (int k = 0; k < kEgB; ++k) any |= (cb + kW * k < C) ? S.nsel[cb + kW * k] : 0;
    for (int j = 0; any && j < NS; ++j) {  // selected tokens leave their clusters, in list order
      const int cj = S.selc[j];
      const int d = cj - cb;
      if (cj < 0 || d < 0 || d >= kW * kEgB || d % kW != 0) continue;  // warp-uniform
      float kf[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        kf[i] = __bfloat162float(j < kEgSelCache ? S.selk[j * kD + 4 * lane + i]
                                                 : Kr[(int64_t)S.selt[j] * kD + 4 * lane + i]);
#pragma unroll
      for (int k = 0; k < kEgB; ++k) {
        if (d == kW * k) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            sk[k][i] = __fsub_rn(sk[k][i], kf[i]);
            sk2[k][i] = __fsub_rn(sk2[k][i], __fmul_rn(kf[i], kf[i]));
          }
        }
      }
    }
    float zd[kEgB], sd[kEgB];
#pragma unroll
    for (int k = 0; k < kEgB; ++k) {
      const int c = cb + kW * k;
      const float inv = c < C ? S.inv[c] : 1.f;
      float kb[4], var[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kb[i] = __fmul_rn(sk[k][i], inv);
        const float p1 = __fmul_rn(sk2[k][i], inv);
        const float p2 = __fmul_rn(kb[i], kb[i]);
        var[i] = fmaxf(__fsub_rn(p1, p2), 0.f);
      }
      zd[k] = warp_tree_dot(qv, kb);
      sd[k] = warp_tree_dot(q2, var);
    }
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < kEgB; ++k) {
        const int c = cb + kW * k;
        if (c < C) {
          S.zd[c] = zd[k];
          S.sd[c] = sd[k];
        }
      }
    }
  }
  __syncthreads();
  float smax = -INFINITY;
  for (int c = tid; c < C; c += NT) {
    const float zbar = __fmul_rn(0.08838834764831845f, S.zd[c]);
    const float s2 = __fmul_rn(0.0078125f, S.sd[c]);
    const float er = erf_f(__fmul_rn(__fsqrt_rn(s2), 0.70710677f));
    const float le = ln_f(fmaxf(er, 1e-30f));
    float sc = __fadd_rn(zbar, S.lg[c]);
    sc = __fadd_rn(sc, __fmul_rn(0.5f, s2));
    sc = __fadd_rn(sc, le);
    S.score[c] = sc;
    smax = fmaxf(smax, S.nt[c] > 1.f ? sc : -INFINITY);
  }
  // ---- water-filling
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, off));
  if (lane == 0) s_red[warp] = smax;
  __syncthreads();
  smax = s_red[0];
#pragma unroll
  for (int v = 1; v < kW; ++v) smax = fmaxf(smax, s_red[v]);
  float tot_part = 0.f;
  for (int c = tid; c < C; c += NT) {
    const bool live = S.nt[c] > 1.f;
    const float w = live ? exp_f(__fsub_rn(S.score[c], smax)) : 0.f;
    const float cap = live ? S.nt[c] : 0.f;
    S.w[c] = w;
    S.cap[c] = cap;
    S.ratio[c] = w > 0.f ? __fdiv_rn(cap, fmaxf(w, 1e-30f)) : INFINITY;
    tot_part = __fadd_rn(tot_part, cap);
  }
  // integer-valued sums (< 2^24): exact in any order, so a block reduction gives the sequential value
  auto block_sum = [&](float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if (lane == 0) s_red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) t = __fadd_rn(t, s_red[w]);
    return t;
  };
  const float tot = block_sum(tot_part);  // its barriers also publish w, cap, ratio, score
  // ranks by (ratio asc, cluster asc) and by (score desc, cluster asc)
  if (C <= 64) {  // one 64-wide warp sort each: warp 0 the ratio order, warp 1 the score order
    if (warp < 2) {
      uint64_t v[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = lane + 32 * h;
        uint32_t key = 0u;
        if (c < C) {
          const float x = warp == 0 ? S.ratio[c] : (S.nt[c] > 1.f ? S.score[c] : -INFINITY);
          key = fkey_eg(x);
          if (warp == 0) key = ~key;  // ascending ratio
        }
        v[h] = c < C ? ((uint64_t)key << 32) | (uint64_t)(0xffffffffu - (uint32_t)c) : 0ull;
      }
      bitonic64_desc(v);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = lane + 32 * h;
        if (e < C) {
          const int c = (int)(0xffffffffu - (uint32_t)v[h]);
          if (warp == 0) {
            S.ord[e] = c;
          } else {
            S.rank2[c] = e;
            S.ord2[e] = c;
          }
        }
      }
    }
  } else {
    for (int c = tid; c < C; c += NT) {
      const float ratio = S.ratio[c];
      const float sm = S.nt[c] > 1.f ? S.score[c] : -INFINITY;
      int r1 = 0, r2 = 0;
      for (int j = 0; j < C; ++j) {
        const float rj = S.ratio[j];
        r1 += (rj < ratio || (rj == ratio && j < c)) ? 1 : 0;
        const float sj = S.nt[j] > 1.f ? S.score[j] : -INFINITY;
        r2 += (sj > sm || (sj == sm && j < c)) ? 1 : 0;
      }
      S.ord[r1] = c;
      S.rank2[c] = r2;
    }
  }
  __syncthreads();
  for (int j = tid; j < C; j += NT) {  // caps, weights and ratios in ratio order
    const int o = S.ord[j];
    S.capo[j] = S.cap[o];
    S.wo[j] = S.w[o];
    S.rato[j] = S.ratio[o];
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefix of the caps in ratio order (integers)
    const int per = (C + 31) / 32;
    const int j0 = lane * per, j1 = min(C, j0 + per);
    float run = 0.f;
    for (int j = j0; j < j1; ++j) run = __fadd_rn(run, S.capo[j]);
    float incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float x = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl = __fadd_rn(incl, x);
    }
    float ex = __fsub_rn(incl, run);
    for (int j = j0; j < j1; ++j) {
      S.cex[j] = ex;
      ex = __fadd_rn(ex, S.capo[j]);
    }
  } else if (warp == 1) {  // suffix sums of the weights in ratio order, accumulated in double from the end
    // every lane runs the same sequential sum over 32 weights held across the warp; lane i keeps the
    // sum that includes weight j0 + i
    double acc = 0.0;
    for (int j0 = (C - 1) & ~31; j0 >= 0; j0 -= 32) {
      const int j = j0 + lane;
      const float wl = j < C ? S.wo[j] : 0.f;
      double mine = 0.0;
#pragma unroll
      for (int i = 31; i >= 0; --i) {
        const float wi = __shfl_sync(0xffffffffu, wl, i);
        if (j0 + i < C) acc = __dadd_rn(acc, (double)wi);
        if (lane == i) mine = acc;
      }
      if (j < C) S.wsuf[j] = __double2float_rn(mine);
    }
  }
  __syncthreads();
  int jj = 0x7fffffff;
  for (int j = tid; j < C; j += NT) {
    const float ws = S.wsuf[j];
    const float f = ws > 0.f ? __fadd_rn(S.cex[j], __fmul_rn(S.rato[j], ws)) : INFINITY;
    if (f >= a.E) jj = min(jj, j);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) jj = min(jj, __shfl_xor_sync(0xffffffffu, jj, off));
  if (lane == 0) s_redi[warp] = jj;
  __syncthreads();
  jj = s_redi[0];
#pragma unroll
  for (int v = 1; v < kW; ++v) jj = min(jj, s_redi[v]);
  if (jj == 0x7fffffff) jj = 0;
  const float lam = __fdiv_rn(__fsub_rn(a.E, S.cex[jj]), fmaxf(S.wsuf[jj], 1e-30f));
  float q_part = 0.f;
  for (int c = tid; c < C; c += NT) {
    float qb = fminf(S.cap[c], floorf(__fmul_rn(lam, S.w[c])));
    if (tot <= a.E) qb = S.cap[c];
    S.qb[c] = qb;
    q_part = __fadd_rn(q_part, qb);
  }
  const float sumq = block_sum(q_part);
  const float rem = fmaxf(__fsub_rn(fminf(tot, a.E), sumq), 0.f);
  // clusters with room, in score order (C <= 64: one bit per rank in two ballots)
  unsigned rb0 = 0u, rb1 = 0u;
  if (C <= 64) {
    const int o0 = lane < C ? S.ord2[lane] : 0, o1 = lane + 32 < C ? S.ord2[lane + 32] : 0;
    rb0 = __ballot_sync(0xffffffffu, lane < C && S.qb[o0] < S.cap[o0]);
    rb1 = __ballot_sync(0xffffffffu, lane + 32 < C && S.qb[o1] < S.cap[o1]);
  }
  for (int c = tid; c < C; c += NT) {  // leftovers: one each to the best-scoring clusters with room
    const int my = S.rank2[c];
    int before = 0;
    if (C <= 64)
      before = my < 32 ? __popc(rb0 & ((1u << my) - 1u)) : __popc(rb0) + __popc(rb1 & ((1u << (my - 32)) - 1u));
    else
      for (int j = 0; j < C; ++j) before += (S.qb[j] < S.cap[j] && S.rank2[j] < my) ? 1 : 0;
    const bool room = S.qb[c] < S.cap[c];
    const float add = (room && (float)before < rem) ? 1.f : 0.f;
    a.quota[rC + c] = __fadd_rn(S.qb[c], add);
    a.nt[rC + c] = S.nt[c];
    a.score[rC + c] = S.score[c];
    if (a.zdot != nullptr) a.zdot[rC + c] = S.zd[c];
  }
}

// ------------------------------------------------------------------------ within-cluster top-q
// One CTA (8 warps) per row.  The row's bf16 score spill is staged in shared memory by one bulk
// copy when it fits (else keys are read from global memory).  Warps take the clusters with q > 0:
// the candidates are the cluster's CSR members (ascending position) followed by its generated
// tokens (the per-cluster list, or a scan of asg over [n0, n) when the list overflowed).
//   q <= 32 and <= 1024 candidates: packed (key, list index) words in registers, q rounds of warp
//     max extraction (ties -> lower list index = lower position), winners sorted by position
//   otherwise: two 8-bit radix passes for the threshold key, then an ordered collection
constexpr int kTqThreads = 256;
constexpr int kTqWarps = kTqThreads / 32;
constexpr int kRegCand = 32;  // candidates per lane in the register path
constexpr int kSmallQ = 32;
constexpr int kU = 4;         // 32-candidate chunks whose loads are issued together (radix path)

struct TopqArgs {
  const uint16_t* scores;
  int64_t sw;
  int Lmax, C, E, rmax, smem_keys;
  const int32_t* mem;
  const int32_t* cstart;
  const int32_t* clen;
  const int32_t* asg;
  const int32_t* reclist;
  const int32_t* reccnt;
  const float* quota;
  const int32_t* n_dev;
  const int32_t* n0_dev;
  int32_t* exp;
  int32_t* status;
};

__device__ __forceinline__ uint32_t ukey16(uint32_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }
// ukey16 of both 16-bit halves of a word
__device__ __forceinline__ uint32_t ukey16x2(uint32_t x) {
  return x ^ ((((x >> 15) & 0x10001u) * 0xffffu) | 0x80008000u);
}

// Register path of top-q for one cluster (one warp): NC member slots per lane, filled with 16-byte
// loads of the member list (lane l holds list words 128 j + 4 l + e, j < NC / 4, relative to the
// 16-byte boundary at or below the list start), plus two slots for generated tokens (up to 64).  Each slot
// holds (ukey16 << 16) | (0xffff - list index), so the maximum is the best score with ties to the
// lower list index (= lower position).  Every lane keeps its own maximum; a round takes the warp
// maximum and only the owning lane rescans its slots.
template <int NC>
__device__ __forceinline__ void topq_regs(const TopqArgs& a, int r, int64_t rc, const int32_t* mp, int nmem,
                                          const int32_t* rec, int ngen, int q, const uint16_t* keys,
                                          int32_t* out, int lane) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(mp);
  const int o = (int)((addr & 15u) >> 2);  // list words before the start inside the first vector
  const int32_t* a0 = mp - o;
  const int32_t* row_end = a.mem + (int64_t)gridDim.x * a.Lmax;
  uint32_t v[NC + 2];
#pragma unroll
  for (int j = 0; j < NC / 4; ++j) {
    const int w = 128 * j + 4 * lane;  // word offset from a0
    const int32_t* p = a0 + w;
    int4 x = make_int4(-1, -1, -1, -1);
    if (w - o < nmem) {
      if (p + 4 <= row_end) {
        x = __ldg(reinterpret_cast<const int4*>(p));
      } else {
        x.x = p + 0 < row_end ? p[0] : -1;
        x.y = p + 1 < row_end ? p[1] : -1;
        x.z = p + 2 < row_end ? p[2] : -1;
        x.w = p + 3 < row_end ? p[3] : -1;
      }
    }
    const int t[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = w + e - o;
      v[4 * j + e] = (idx >= 0 && idx < nmem) ? (ukey16(keys[t[e]]) << 16) | (uint32_t)(0xffff - idx) : 0u;
    }
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int gi = lane + 32 * g;
    v[NC + g] = gi < ngen ? (ukey16(keys[rec[gi]]) << 16) | (uint32_t)(0xffff - (nmem + gi)) : 0u;
  }
  uint32_t lm = 0u;
#pragma unroll
  for (int i = 0; i < NC + 2; ++i) lm = max(lm, v[i]);
  int my_idx = 0x7fffffff;  // list index of the winner this lane records (lane k <-> k-th winner)
  for (int k = 0; k < q; ++k) {
    uint32_t wm = lm;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, off));
    if (wm == 0u) break;
    if (lm == wm) {  // the unique owner drops it and rescans
      uint32_t nm = 0u;
#pragma unroll
      for (int i = 0; i < NC + 2; ++i) {
        v[i] = v[i] == wm ? 0u : v[i];
        nm = max(nm, v[i]);
      }
      lm = nm;
    }
    if (lane == k) my_idx = 0xffff - (int)(wm & 0xffffu);
  }
  int rank = 0;
  for (int j = 0; j < q; ++j) {
    const int oth = __shfl_sync(0xffffffffu, my_idx, j);
    rank += (oth < my_idx) ? 1 : 0;
  }
  if (lane < q && my_idx != 0x7fffffff) out[rank] = my_idx < nmem ? mp[my_idx] : rec[my_idx - nmem];
}

__global__ void __launch_bounds__(kTqThreads, 3) topq_kernel(const TopqArgs a) {
  extern __shared__ __align__(128) uint16_t s_spill[];  // the row's scores (when a.smem_keys)
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int s_base[kMaxC + 1];
  __shared__ int s_q[kMaxC];
  __shared__ int s_next;
  __shared__ int s_hist[kTqWarps][256];
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = a.C;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  const uint16_t* sr = a.scores + (int64_t)r * a.sw;
  const uint32_t bar = smem_u32(&mbar);
  const int nbytes = ((min(n, a.Lmax) + 7) & ~7) * 2;
  if (tid == 0) {
    mbar_init(bar);
    if (a.smem_keys && nbytes > 0) bulk_load(s_spill, sr, (uint32_t)nbytes, bar);
    s_next = 0;
  }
  for (int c = tid; c < C; c += kTqThreads) s_q[c] = quota_int(a.quota[(int64_t)r * C + c], a.E);
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      s_base[c] = run;
      run += s_q[c];
    }
    s_base[C] = run;
  }
  __syncthreads();
  int32_t* out = a.exp + (int64_t)r * a.E;
  for (int i = s_base[C] + tid; i < a.E; i += kTqThreads) out[i] = -1;
  const bool ok = !(a.smem_keys && nbytes > 0) || mbar_wait(bar, 0);
  if (!__syncthreads_and(ok)) {
    if (tid == 0 && a.status != nullptr) atomicExch(a.status, 4);
    if (!ok) mbar_wait(bar, 0);
    return;
  }
  const uint16_t* keys = a.smem_keys ? s_spill : sr;
  const int32_t* asg_r = a.asg + (int64_t)r * a.Lmax;
  int* hist = s_hist[warp];
  const unsigned lt = (1u << lane) - 1u;
  while (true) {
    int c = 0;
    if (lane == 0) {
      do {
        c = atomicAdd(&s_next, 1);
      } while (c < C && s_q[c] <= 0);
    }
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= C) break;
    const int q = s_q[c], base = s_base[c];
    const int64_t rc = (int64_t)r * C + c;
    const int nmem = a.clen[rc];
    const int32_t* mp = a.mem + (int64_t)r * a.Lmax + a.cstart[rc];
    const int cnt = a.reclist ? a.reccnt[rc] : 0x7fffffff;
    const bool use_list = a.reclist != nullptr && cnt <= a.rmax;
    const int32_t* rec = use_list ? a.reclist + rc * a.rmax : nullptr;
    const int ngen = use_list ? cnt : 0;
    if (use_list && q <= kSmallQ && ngen <= 64 && nmem + 3 <= 32 * kRegCand) {
      const int span = nmem + 3;
      if (span <= 256)
        topq_regs<8>(a, r, rc, mp, nmem, rec, ngen, q, keys, out + base, lane);
      else if (span <= 512)
        topq_regs<16>(a, r, rc, mp, nmem, rec, ngen, q, keys, out + base, lane);
      else
        topq_regs<32>(a, r, rc, mp, nmem, rec, ngen, q, keys, out + base, lane);
      continue;
    }
    // ---- radix path: candidates enumerated in order (members, then generated tokens)
    const int ngen_scan = max(0, n - n0);
    auto for_each = [&](auto&& f) {
      for (int i0 = 0; i0 < nmem; i0 += 32 * kU) {
        int t[kU];
        bool v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + 32 * u + lane;
          v[u] = i < nmem;
          t[u] = v[u] ? mp[i] : 0;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (i0 + 32 * u < nmem) f(v[u], t[u], v[u] ? ukey16(keys[t[u]]) : 0u);
      }
      if (use_list) {
        for (int i0 = 0; i0 < cnt; i0 += 32) {
          const int i = i0 + lane;
          const bool v = i < cnt;
          const int t = v ? rec[i] : 0;
          f(v, t, v ? ukey16(keys[t]) : 0u);
        }
      } else {
        for (int i0 = 0; i0 < ngen_scan; i0 += 32) {
          const int t = n0 + i0 + lane;
          const bool v = (i0 + lane < ngen_scan) && asg_r[t] == c;
          f(v, t, v ? ukey16(keys[t]) : 0u);
        }
      }
    };
    int above = 0, hi = 0, lo = 0;
    bool all = false;
    for (int pass = 0; pass < 2 && !all; ++pass) {
      for (int b = lane; b < 256; b += 32) hist[b] = 0;
      __syncwarp();
      for_each([&](bool v, int t, uint32_t k) {
        if (v && (pass == 0 || (int)(k >> 8) == hi)) atomicAdd(&hist[pass == 0 ? (k >> 8) : (k & 255)], 1);
      });
      __syncwarp();
      int cnt8[8], sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt8[i] = hist[255 - 8 * lane - i];
        sum += cnt8[i];
      }
      int incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const int excl = incl - sum;
      const int need = q - above;
      int fb = -1, fa = 0;
      if (excl < need && incl >= need) {
        int run = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (fb < 0 && run + cnt8[i] >= need) {
            fb = 255 - 8 * lane - i;
            fa = run;
          }
          run += cnt8[i];
        }
      }
      const unsigned who = __ballot_sync(0xffffffffu, fb >= 0);
      if (who == 0u) {
        all = true;  // fewer candidates than q: take every one
      } else {
        const int src = __ffs(who) - 1;
        const int d = __shfl_sync(0xffffffffu, fb, src);
        above += __shfl_sync(0xffffffffu, fa, src);
        if (pass == 0) hi = d;
        else lo = d;
      }
      __syncwarp();
    }
    const uint32_t T = all ? 0u : (((uint32_t)hi << 8) | (uint32_t)lo);
    const int need_eq = all ? 0 : q - above;
    int taken = 0, ties = 0;
    for_each([&](bool v, int t, uint32_t k) {
      const bool gt = v && k > T;
      const bool eq = v && k == T;
      const unsigned beq = __ballot_sync(0xffffffffu, eq);
      const bool take = gt || (eq && ties + __popc(beq & lt) < need_eq);
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      const int slot = taken + __popc(bt & lt);
      if (take && slot < q) out[base + slot] = t;
      taken += __popc(bt);
      ties += __popc(beq);
    });
    __syncwarp();
  }
}

// ------------------------------------------------------------------------ top-q, streamed member keys
// Persistent variant of top-q with one key buffer, for rows of about 35K to 47K positions (shorter
// rows take topq_pipe_kernel): one CTA of 32 warps per SM walks rows r = blockIdx.x, + gridDim.x, ...
// Per row:
//   phase 1: the whole CSR member list of the row is streamed with 16-byte loads (every thread has
//            several in flight) and turned into a contiguous array of 16-bit score keys in CSR order
//            (the score row itself was staged by a bulk copy); keys of generated positions [n0, n)
//            are staged too;
//   phase 2: warps take the clusters with q > 0 and select from contiguous shared-memory keys
//            (streamed path: (key, list index) words, q rounds of warp maximum; radix path for
//            larger quotas); winners are recorded in shared memory as CSR slots (or positions of
//            generated tokens) and turned into positions by one parallel pass over the row.
// While phase 2 runs, the next row's score row is already being copied into the freed buffer.
constexpr int kTsThreads = 1024;
constexpr int kTsWarps = kTsThreads / 32;
constexpr int kTsGenCap = 4096;  // generated positions whose keys are staged
constexpr int kTsU = 8;          // 16-byte member vectors a thread has in flight in phase 1

struct TsRow {
  const uint16_t* key;   // member keys of the row, CSR order (key[i] = member i; key - mo is 8-byte aligned)
  const uint16_t* gkey;  // keys of positions n0 .. n0 + gcount - 1
  const uint16_t* sr;    // the row's score bits in global memory
  const int32_t* mrow;   // the row's member list in global memory
  int n0, nsp, gcount, mo;
};

__device__ __forceinline__ uint32_t ts_key_at(const TsRow& w, int t) {
  if (t < 0 || t >= w.nsp) return 0u;
  if (t >= w.n0 && t - w.n0 < w.gcount) return w.gkey[t - w.n0];
  return ukey16(w.sr[t]);
}

// Winner encodings in the row's shared-memory list: a CSR slot (>= 0) of a member, or -(position+1)
// of a generated token.
__device__ __forceinline__ int ts_enc(int idx, int cs, int nmem, const int32_t* rec) {
  return idx < nmem ? cs + idx : -(rec[idx - nmem] + 1);
}

template <int NC>
__device__ __forceinline__ void topq_keys_regs(const TsRow& w, int cs, int nmem, const int32_t* rec, int ngen,
                                               int q, int* win, int lim, int lane) {
  const int o = (cs + w.mo) & 3, a0 = cs - o;  // w.key + a0 is 8-byte aligned
  uint32_t v[NC + 2];
#pragma unroll
  for (int j = 0; j < NC / 4; ++j) {
    const int wd = 128 * j + 4 * lane;
    const uint2 x = *reinterpret_cast<const uint2*>(w.key + a0 + wd);
    const uint32_t k4[4] = {x.x & 0xffffu, x.x >> 16, x.y & 0xffffu, x.y >> 16};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = wd + e - o;
      v[4 * j + e] = (idx >= 0 && idx < nmem) ? (k4[e] << 16) | (uint32_t)(0xffff - idx) : 0u;
    }
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int gi = lane + 32 * g;
    v[NC + g] = gi < ngen ? (ts_key_at(w, rec[gi]) << 16) | (uint32_t)(0xffff - (nmem + gi)) : 0u;
  }
  // lane-local best two; a lane gives up its values in decreasing order, so the values it still holds
  // are exactly those below the last one it gave up (words are unique)
  uint32_t m1 = 0u, m2 = 0u;
#pragma unroll
  for (int i = 0; i < NC + 2; ++i) {
    m2 = max(m2, min(m1, v[i]));
    m1 = max(m1, v[i]);
  }
  bool have2 = true;  // m2 is this lane's second best
  int my_idx = 0x7fffffff;
  for (int k = 0; k < q; ++k) {
    const uint32_t wm = __reduce_max_sync(0xffffffffu, m1);
    if (wm == 0u) break;
    if (m1 == wm) {  // the unique owner
      if (have2) {
        m1 = m2;
        have2 = false;
      } else {  // rescan below the value just taken
        m1 = 0u;
        m2 = 0u;
#pragma unroll
        for (int i = 0; i < NC + 2; ++i) {
          const uint32_t c = v[i] < wm ? v[i] : 0u;
          m2 = max(m2, min(m1, c));
          m1 = max(m1, c);
        }
        have2 = true;
      }
    }
    if (lane == k) my_idx = 0xffff - (int)(wm & 0xffffu);
  }
  int rank = 0;
  for (int j = 0; j < q; ++j) {
    const int oth = __shfl_sync(0xffffffffu, my_idx, j);
    rank += (oth < my_idx) ? 1 : 0;
  }
  if (lane < q && my_idx != 0x7fffffff && rank < lim) win[rank] = ts_enc(my_idx, cs, nmem, rec);
}

// The same selection without a register copy of the cluster: each lane streams its keys (four per
// 8-byte word, words 128 keys apart) from shared memory once to find its best two, and the lane that
// gives up its second best re-reads its keys below the value just taken.  Only (m1, m2) live in
// registers, so the kernels run 24 or 32 warps per SM and any cluster size takes this path.  Words whose
// four keys all lie inside the cluster for every lane (all but the first and the last one or two)
// skip the bounds tests and build their (key, 0xffff - index) words with byte permutes from a packed
// pair of index complements.
template <bool FILTER>
__device__ __forceinline__ void ts_best2(const uint16_t* kb, int idx0, int nmem, int nj, int j_lo, int j_hi,
                                         uint32_t (&g)[2], const TsRow& w, const int (&gt)[2], int lane,
                                         uint32_t below, uint32_t& m1, uint32_t& m2) {
  m1 = 0u;
  m2 = 0u;
  auto take = [&](uint32_t c) {
    if (FILTER) c = c < below ? c : 0u;
    m2 = max(m2, min(m1, c));
    m1 = max(m1, c);
  };
  auto checked = [&](int j) {
    const uint2 x = *reinterpret_cast<const uint2*>(kb + 128 * j);
    const uint32_t k4[4] = {x.x << 16, x.x & 0xffff0000u, x.y << 16, x.y & 0xffff0000u};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = idx0 + 128 * j + e;
      take((uint32_t)idx < (uint32_t)nmem ? k4[e] | (uint32_t)(0xffff - idx) : 0u);
    }
  };
  for (int j = 0; j < min(j_lo, nj); ++j) checked(j);
  // interior words: index complements of keys 0,1 and 2,3 as packed 16-bit pairs (all >= 0 here, so
  // the packed subtraction never borrows across the halves)
  const uint32_t b0 = (uint32_t)(0xffff - (idx0 + 128 * j_lo)), b2 = b0 - 2u;
  const uint32_t p01 = (b0 & 0xffffu) | ((b0 - 1u) << 16), p23 = (b2 & 0xffffu) | ((b2 - 1u) << 16);
#pragma unroll 1
  for (int j = j_lo; j < j_hi; ++j) {
    const uint2 x = *reinterpret_cast<const uint2*>(kb + 128 * j);
    const uint32_t dj = (uint32_t)(128 * (j - j_lo)) * 0x10001u;
    const uint32_t l01 = p01 - dj, l23 = p23 - dj;
    take(__byte_perm(x.x, l01, 0x1054));  // key 0 over the low complement
    take(__byte_perm(x.x, l01, 0x3276));  // key 1 over the high complement
    take(__byte_perm(x.y, l23, 0x1054));
    take(__byte_perm(x.y, l23, 0x3276));
  }
  for (int j = max(j_hi, j_lo); j < nj; ++j) checked(j);
  if (!FILTER) {  // the generated candidates' words, from list entries loaded before the member pass
#pragma unroll
    for (int h = 0; h < 2; ++h)
      g[h] = gt[h] >= 0 ? (ts_key_at(w, gt[h]) << 16) | (uint32_t)(0xffff - (nmem + lane + 32 * h)) : 0u;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) take(g[h]);
}

__device__ __forceinline__ void topq_keys_stream(const TsRow& w, int cs, int nmem, const int32_t* rec, int ngen,
                                                 int q, int* win, int lim, int lane) {
  const int o = (cs + w.mo) & 3;
  const uint16_t* kb = w.key + (cs - o) + 4 * lane;  // 8-byte aligned
  const int nj = (nmem + o + 127) >> 7;              // words a lane reads
  const int idx0 = 4 * lane - o;                     // list index of the lane's first key
  const int j_lo = o > 0 ? 1 : 0;                    // first word inside the cluster for every lane
  const int j_hi = (nmem + o) >> 7;                  // words [j_lo, j_hi) lie inside for every lane
  uint32_t g[2];
  int gt[2];  // generated positions of this lane's candidates, loaded now, used after the member pass
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gi = lane + 32 * h;
    gt[h] = gi < ngen ? rec[gi] : -1;
  }
  uint32_t m1, m2;
  ts_best2<false>(kb, idx0, nmem, nj, j_lo, j_hi, g, w, gt, lane, 0u, m1, m2);
  bool have2 = true;  // m2 is this lane's second best
  int my_idx = 0x7fffffff;
  for (int k = 0; k < q; ++k) {
    const uint32_t wm = __reduce_max_sync(0xffffffffu, m1);
    if (wm == 0u) break;
    if (m1 == wm) {  // the unique owner
      if (have2) {
        m1 = m2;
        have2 = false;
      } else {  // re-read below the value just taken
        ts_best2<true>(kb, idx0, nmem, nj, j_lo, j_hi, g, w, gt, lane, wm, m1, m2);
        have2 = true;
      }
    }
    if (lane == k) my_idx = 0xffff - (int)(wm & 0xffffu);
  }
  int rank = 0;
  for (int j = 0; j < q; ++j) {
    const int oth = __shfl_sync(0xffffffffu, my_idx, j);
    rank += (oth < my_idx) ? 1 : 0;
  }
  if (lane < q && my_idx != 0x7fffffff && rank < lim) win[rank] = ts_enc(my_idx, cs, nmem, rec);
}

// Row metadata of one work item in shared memory: quotas, CSR starts and lengths, generated-list
// counts, the order in which warps take the clusters, and the exclusive prefix of the quotas (C + 1).
struct TsMeta {
  int *q, *cs, *cl, *rcnt, *ord, *base;
};

__device__ __forceinline__ void ts_load_meta(const TopqArgs& a, const TsMeta& m, int row, int tid, int nthreads) {
  const int64_t rc0 = (int64_t)row * a.C;
  for (int c = tid; c < a.C; c += nthreads) {
    m.q[c] = quota_int(a.quota[rc0 + c], a.E);
    m.cs[c] = a.cstart[rc0 + c];
    m.cl[c] = a.clen[rc0 + c];
    m.rcnt[c] = a.reclist ? a.reccnt[rc0 + c] : 0x7fffffff;
  }
}

// One warp: the exclusive prefix of the quotas and the order in which warps take the clusters.
__device__ __forceinline__ void ts_prefix(const TsMeta& m, int C, int lane) {
  const int per = (C + 31) / 32;
  const int c0 = lane * per, c1 = min(C, c0 + per);
  int run = 0;
  for (int c = c0; c < c1; ++c) run += m.q[c];
  int incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += x;
  }
  int ex = incl - run;
  for (int c = c0; c < c1; ++c) {
    m.base[c] = ex;
    ex += m.q[c];
  }
  if (lane == 31) m.base[C] = incl;
  // Largest clusters first (C <= 64), so that the last clusters taken are short ones and the
  // warps reach the end-of-row barrier together; clusters with q = 0 go last.
  if (C <= 64) {
    uint64_t wv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = lane + 32 * h;
      uint32_t work = 0u;
      if (c < C && m.q[c] > 0)  // clusters for the radix path (quota above 32) cost the most per key: first
        work = (m.q[c] > kSmallQ ? 0x100000u : 0u) + 1u + (uint32_t)m.cl[c] + (uint32_t)min(m.rcnt[c], 4096);
      wv[h] = c < C ? ((uint64_t)work << 32) | (uint64_t)(0xffffffffu - (uint32_t)c) : 0ull;
    }
    bitonic64_desc(wv);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      if (e < C) m.ord[e] = (int)(0xffffffffu - (uint32_t)wv[h]);
    }
  } else {
    for (int c = lane; c < C; c += 32) m.ord[c] = c;
  }
}

// One lane keys U 16-byte vectors of the member list (vectors vbase, vbase + vstride, ...): the four
// positions of a vector become four score keys in one 8-byte store at key slot 4 * vector.  All loads
// are issued before the first gather from the staged score row.
template <int U>
__device__ __forceinline__ void ts_key_vecs(const int32_t* m0, const int32_t* mem_end, int vbase, int vstride,
                                            int nvec, const uint16_t* s_spill, uint32_t lim, uint16_t* s_key) {
  int4 x[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int vi = vbase + u * vstride;
    const int32_t* p = m0 + 4 * vi;
    x[u] = make_int4(0, 0, 0, 0);
    if (vi < nvec) {
      if (p + 4 <= mem_end) {
        x[u] = __ldg(reinterpret_cast<const int4*>(p));
      } else {
        x[u].x = p + 0 < mem_end ? p[0] : 0;
        x[u].y = p + 1 < mem_end ? p[1] : 0;
        x[u].z = p + 2 < mem_end ? p[2] : 0;
        x[u].w = p + 3 < mem_end ? p[3] : 0;
      }
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int vi = vbase + u * vstride;
    if (vi < nvec) {  // list entries are positions; the clamp keeps the reads inside the staged row
      const uint32_t k0 = s_spill[min((uint32_t)x[u].x, lim)], k1 = s_spill[min((uint32_t)x[u].y, lim)];
      const uint32_t k2 = s_spill[min((uint32_t)x[u].z, lim)], k3 = s_spill[min((uint32_t)x[u].w, lim)];
      *reinterpret_cast<uint2*>(s_key + 4 * vi) = make_uint2(ukey16x2(k0 | (k1 << 16)), ukey16x2(k2 | (k3 << 16)));
    }
  }
}

// Selection of one work item: the warps of the CTA take its clusters with q > 0 in [c_lo, c_hi) from
// the shared counter *next and write each cluster's winners (CSR slots, or -(position + 1) of
// generated tokens) at its quota offset in s_win.  Small quotas with short generated lists take the
// streamed register path; the rest the radix path (two 8-bit histogram passes for the threshold key,
// then an ordered collection).
// The radix path of the selection (quota above the register path's 32, or a long generated list):
// two 8-bit histogram passes over the cluster's keys for the threshold key, then an ordered
// collection.
__device__ __forceinline__ void ts_radix(const TsRow w, int E, int c, int q, int base, int cs, int nmem,
                                      const int32_t* rec, bool use_list, int cnt, int n, int n0,
                                      const int32_t* asg_r, int* s_win, uint32_t* hist, int lane) {
  const unsigned lt = (1u << lane) - 1u;
  // radix path over (list index, key): members from the key array, then generated tokens
  const int ngen_scan = max(0, n - n0);
  auto enc_of = [&](int idx) -> int {
    if (idx < nmem) return cs + idx;
    return -((use_list ? rec[idx - nmem] : n0 + (idx - nmem)) + 1);
  };
  auto for_each = [&](auto&& f) {
    for (int i0 = 0; i0 < nmem; i0 += 32) {
      const int i = i0 + lane;
      const bool v = i < nmem;
      f(v, i, v ? (uint32_t)w.key[cs + i] : 0u);
    }
    if (use_list) {
      for (int i0 = 0; i0 < cnt; i0 += 32) {
        const int i = i0 + lane;
        const bool v = i < cnt;
        f(v, nmem + i, v ? ts_key_at(w, rec[i]) : 0u);
      }
    } else {
      for (int i0 = 0; i0 < ngen_scan; i0 += 32) {
        const int t = n0 + i0 + lane;
        const bool v = (i0 + lane < ngen_scan) && asg_r[t] == c;
        f(v, nmem + i0 + lane, v ? ts_key_at(w, t) : 0u);
      }
    }
  };
  int above = 0, hi = 0, lo = 0;
  bool all = false;
  for (int pass = 0; pass < 2 && !all; ++pass) {
    for (int b = lane; b < 128; b += 32) hist[b] = 0u;
    __syncwarp();
    for_each([&](bool v, int, uint32_t k) {
      if (v && (pass == 0 || (int)(k >> 8) == hi)) {
        const uint32_t d = pass == 0 ? (k >> 8) : (k & 255u);
        atomicAdd(&hist[d >> 1], 1u << (16 * (d & 1u)));
      }
    });
    __syncwarp();
    int cnt8[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = 255 - 8 * lane - i;
      cnt8[i] = (int)((hist[d >> 1] >> (16 * (d & 1))) & 0xffffu);
      sum += cnt8[i];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += x;
    }
    const int excl = incl - sum;
    const int need = q - above;
    int fb = -1, fa = 0;
    if (excl < need && incl >= need) {
      int run = excl;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (fb < 0 && run + cnt8[i] >= need) {
          fb = 255 - 8 * lane - i;
          fa = run;
        }
        run += cnt8[i];
      }
    }
    const unsigned who = __ballot_sync(0xffffffffu, fb >= 0);
    if (who == 0u) {
      all = true;
    } else {
      const int src = __ffs(who) - 1;
      const int d = __shfl_sync(0xffffffffu, fb, src);
      above += __shfl_sync(0xffffffffu, fa, src);
      if (pass == 0) hi = d;
      else lo = d;
    }
    __syncwarp();
  }
  const uint32_t T = all ? 0u : (((uint32_t)hi << 8) | (uint32_t)lo);
  const int need_eq = all ? 0 : q - above;
  int taken = 0, ties = 0;
  for_each([&](bool v, int idx, uint32_t k) {
    const bool gt = v && k > T;
    const bool eq = v && k == T;
    const unsigned beq = __ballot_sync(0xffffffffu, eq);
    const bool take = gt || (eq && ties + __popc(beq & lt) < need_eq);
    const unsigned bt = __ballot_sync(0xffffffffu, take);
    const int slot = taken + __popc(bt & lt);
    if (take && slot < q && base + slot < E) s_win[base + slot] = enc_of(idx);
    taken += __popc(bt);
    ties += __popc(beq);
  });
  __syncwarp();
}

__device__ __forceinline__ void ts_select(const TopqArgs& a, const TsRow& w, const TsMeta& m, int r, int c_lo,
                                          int c_hi, int n, int n0, int* next, int* s_win, uint32_t* hist,
                                          int lane) {
  const int C = a.C;
  const int64_t rC = (int64_t)r * C;
  const int32_t* asg_r = a.asg + (int64_t)r * a.Lmax;
  while (true) {
    int c = C;
    if (lane == 0) {
      int i;
      do {
        i = atomicAdd(next, 1);
        c = i < C ? m.ord[i] : C;
      } while (c < C && (m.q[c] <= 0 || c < c_lo || c >= c_hi));
    }
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= C) break;
    const int q = m.q[c], base = m.base[c], cs = m.cs[c], nmem = m.cl[c];
    const int cnt = m.rcnt[c];
    const bool use_list = a.reclist != nullptr && cnt <= a.rmax;
    const int32_t* rec = use_list ? a.reclist + (rC + c) * a.rmax : nullptr;
    const int ngen = use_list ? cnt : 0;
    if (use_list && q <= kSmallQ && ngen <= 64 && nmem + ngen < 0xffff) {
      topq_keys_stream(w, cs, nmem, rec, ngen, q, s_win + base, a.E - base, lane);
      continue;
    }
    ts_radix(w, a.E, c, q, base, cs, nmem, rec, use_list, cnt, n, n0, asg_r, s_win, hist, lane);
  }
}

// parts > 1 (fewer rows than SMs): work item w is row w / parts, clusters [p C / parts, (p+1) C / parts)
// of it for p = w % parts; each item's CTA stages the whole score row but keys and selects only its
// clusters' members (their CSR range), so a row's work is spread over `parts` SMs.
__global__ void __launch_bounds__(kTsThreads, 1) topq_stream_kernel(const TopqArgs a, int R, int spill_cap,
                                                                    int key_cap, int parts) {
  extern __shared__ __align__(128) unsigned char ts_smem[];
  uint16_t* s_spill = reinterpret_cast<uint16_t*>(ts_smem);
  uint16_t* s_key = reinterpret_cast<uint16_t*>(ts_smem + spill_cap);
  uint16_t* s_gkey = s_key + key_cap;
  int* s_win = reinterpret_cast<int*>(s_gkey + kTsGenCap);  // a.E winner encodings
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int s_base_[2][kMaxC + 1];  // row metadata, double-buffered: the next row's loads while
  __shared__ int s_q_[2][kMaxC], s_cs_[2][kMaxC], s_cl_[2][kMaxC], s_rcnt_[2][kMaxC];  // this row runs
  __shared__ int s_ord_[2][kMaxC];  // the order in which warps take the clusters
  __shared__ int s_next;
  __shared__ uint32_t s_hist[kTsWarps][128];  // radix path: 256 16-bit counts per warp, two to a word
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = a.C;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  const int nsp = min(n, a.Lmax);
  const uint32_t nbytes = (uint32_t)((nsp + 7) & ~7) * 2u;
  const int gcount = min(max(0, nsp - n0), kTsGenCap);
  const uint32_t bar = smem_u32(&mbar);
  const int32_t* mem_end = a.mem + (int64_t)R * a.Lmax;
  auto meta = [&](int set) {
    return TsMeta{s_q_[set], s_cs_[set], s_cl_[set], s_rcnt_[set], s_ord_[set], s_base_[set]};
  };
  auto winners_out = [&](int row, int lo, int hi) {  // CSR slots / generated positions -> positions
    int32_t* pout = a.exp + (int64_t)row * a.E;
    const int32_t* pm = a.mem + (int64_t)row * a.Lmax;
    for (int i = lo + tid; i < hi; i += kTsThreads) {
      const int e = s_win[i];
      pout[i] = e >= 0 ? pm[e] : -e - 1;
    }
  };
  const int W = R * parts;  // work items
  if (tid == 0) {
    mbar_init(bar);
    if (nbytes) bulk_load(s_spill, a.scores + (int64_t)(blockIdx.x / parts) * a.sw, nbytes, bar);
  }
  ts_load_meta(a, meta(0), blockIdx.x / parts, tid, kTsThreads);
  __syncthreads();
  if (warp == 0) ts_prefix(meta(0), C, lane);
  int it = 0, cur = 0, prev_r = -1, prev_lo = 0, prev_hi = 0;
  for (int wi = blockIdx.x; wi < W; wi += gridDim.x, ++it, cur ^= 1) {
    const int r = wi / parts, part = wi - r * parts;
    const int nwi = wi + (int)gridDim.x;
    const int nr = nwi < W ? nwi / parts : R;  // the next item's row (R: none)
    const int c_lo = part * C / parts, c_hi = (part + 1) * C / parts;
    const int* s_cs = s_cs_[cur];
    const int* s_cl = s_cl_[cur];
    const int* s_base = s_base_[cur];
    const bool ok = nbytes == 0 || mbar_wait(bar, (uint32_t)(it & 1));
    if (!__syncthreads_and(ok)) {
      if (tid == 0 && a.status != nullptr) atomicExch(a.status, 4);
      if (!ok) mbar_wait(bar, (uint32_t)(it & 1));  // let the copy in flight land before leaving
      return;
    }
    // overlapping phase 1: the previous row's winner positions, the next row's metadata, this row's pads
    if (prev_r >= 0) winners_out(prev_r, prev_lo, prev_hi);
    if (nr < R) ts_load_meta(a, meta(cur ^ 1), nr, tid, kTsThreads);
    int32_t* out = a.exp + (int64_t)r * a.E;
    if (part == 0)
      for (int i = s_base[C] + tid; i < a.E; i += kTsThreads) out[i] = -1;
    if (tid == 0) s_next = 0;
    // ---- phase 1: member keys in CSR order (key slot = member index + mo, so every 16-byte vector of
    // the member list becomes one 8-byte store of four keys), generated-position keys
    const int m_lo = s_cs[c_lo], m_hi = s_cs[c_hi - 1] + s_cl[c_hi - 1];  // this item's members
    const int32_t* mrow = a.mem + (int64_t)r * a.Lmax;
    const int mo = (int)((reinterpret_cast<uintptr_t>(mrow) & 15u) >> 2);
    const int32_t* m0 = mrow - mo;
    const int nvec = (m_hi + mo + 3) >> 2;
    const uint32_t lim = (uint32_t)(spill_cap / 2 - 1);  // list entries are positions; clamp keeps reads inside
    for (int v0 = ((m_lo + mo) >> 2) + tid; v0 < nvec; v0 += kTsThreads * kTsU)
      ts_key_vecs<kTsU>(m0, mem_end, v0, kTsThreads, nvec, s_spill, lim, s_key);
    for (int i = tid; i < gcount; i += kTsThreads) s_gkey[i] = (uint16_t)ukey16(s_spill[n0 + i]);
    __syncthreads();
    if (tid == 0 && nr < R && nbytes) {  // the staged row is free: fetch the next one
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bulk_load(s_spill, a.scores + (int64_t)nr * a.sw, nbytes, bar);
    }
    if (warp == 0 && nr < R) ts_prefix(meta(cur ^ 1), C, lane);
    // ---- phase 2: clusters with q > 0
    TsRow w{s_key + mo, s_gkey, a.scores + (int64_t)r * a.sw, mrow, n0, nsp, gcount, mo};
    ts_select(a, w, meta(cur), r, c_lo, c_hi, n, n0, &s_next, s_win, s_hist[warp], lane);
    __syncthreads();  // winners complete; keys and the cluster counter are reused by the next row
    prev_r = r;
    prev_lo = min(s_base[c_lo], a.E);
    prev_hi = min(s_base[c_hi], a.E);
  }
  if (prev_r >= 0) winners_out(prev_r, prev_lo, prev_hi);
}

// ------------------------------------------------------------------------ top-q, pipelined rows
// The persistent top-q with each work item's keying overlapped with the previous item's selection.
// Shared memory holds one staged score row, two key buffers, two winner lists and three metadata
// sets.  In iteration i most warps first take clusters of item i until none is left, then take
// chunks of item i + 1's member list (32 x kTpU vectors, 512 members) from a second counter and
// key them from the staged score row of item i + 1; kTpKeyFirst warps do the same in the other
// order.  So keying and selection run side by side, and the warps that finish one job early help
// with the other.  One CTA barrier per item; after it the score row of item i + 2 is
// fetched into the freed buffer while item i + 1 is selected.  Keys of generated positions [n0, n)
// are keyed too, into the key buffer's slots past the members.
constexpr int kTpThreads = 768;
constexpr int kTpWarps = kTpThreads / 32;
constexpr int kTpU = 4;  // 16-byte member vectors per lane in one keying chunk (512 members)
// Warps that key the next item before selecting (the rest select first).
constexpr int kTpKeyFirst = 9;

__global__ void __launch_bounds__(kTpThreads, 1) topq_pipe_kernel(const TopqArgs a, int R, int spill_cap,
                                                                  int key_cap, int parts) {
  extern __shared__ __align__(128) unsigned char tp_smem[];
  const int C = a.C, E = a.E;
  const int W = R * parts;  // work items
  if ((int)blockIdx.x >= W) return;
  uint16_t* s_spill = reinterpret_cast<uint16_t*>(tp_smem);
  uint16_t* s_key0 = reinterpret_cast<uint16_t*>(tp_smem + spill_cap);  // two buffers of key_cap keys
  int* s_win0 = reinterpret_cast<int*>(s_key0 + 2 * key_cap);            // two lists of E winners
  int* s_meta = s_win0 + 2 * E;                                          // three sets of 6 C + 1 ints
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int s_next[2], s_kc[2];  // cluster counters (selection), chunk counters (keying)
  __shared__ uint32_t s_hist[kTpWarps][128];  // radix path: 256 16-bit counts per warp, two to a word
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = (int)gridDim.x;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  const int nsp = min(n, a.Lmax);
  const uint32_t nbytes = (uint32_t)((nsp + 7) & ~7) * 2u;
  const uint32_t bar = smem_u32(&mbar);
  const int32_t* mem_end = a.mem + (int64_t)R * a.Lmax;
  const uint32_t lim = (uint32_t)(spill_cap / 2 - 1);  // list entries are positions; the clamp keeps reads inside
  auto meta = [&](int set) {
    int* p = s_meta + set * (6 * C + 1);
    return TsMeta{p, p + C, p + 2 * C, p + 3 * C, p + 4 * C, p + 5 * C};
  };
  auto mrow_of = [&](int r) { return a.mem + (int64_t)r * a.Lmax; };
  auto mo_of = [&](const int32_t* mrow) { return (int)((reinterpret_cast<uintptr_t>(mrow) & 15u) >> 2); };
  // keying of work item wi into kbuf (key slot = member index + mo): chunks from the counter *cnt
  auto key_item = [&](int wi, uint16_t* kbuf, int* cnt, const TsMeta& m) {
    const int r = wi / parts, part = wi - r * parts;
    const int c_lo = part * C / parts, c_hi = (part + 1) * C / parts;
    const int m_lo = m.cs[c_lo], m_hi = m.cs[c_hi - 1] + m.cl[c_hi - 1];
    const int32_t* mrow = mrow_of(r);
    const int mo = mo_of(mrow);
    const int nvec = (m_hi + mo + 3) >> 2;
    const int vb0 = (m_lo + mo) >> 2;
    while (true) {
      int ch = 0;
      if (lane == 0) ch = atomicAdd(cnt, 1);
      ch = __shfl_sync(0xffffffffu, ch, 0);
      const int vb = vb0 + ch * (32 * kTpU);
      if (vb >= nvec) break;
      ts_key_vecs<kTpU>(mrow - mo, mem_end, vb + lane, 32, nvec, s_spill, lim, kbuf);
    }
    // keys of the generated positions [n0, n) in the slots past the members' last 4-key vector (every
    // warp keys its share)
    const int gbase = (mo + max(n0, m_hi) + 3) & ~3;
    const int gcnt = max(0, min(nsp - n0, key_cap - gbase));
    for (int g = warp * 32 + lane; g < gcnt; g += kTpThreads) kbuf[gbase + g] = (uint16_t)ukey16(s_spill[n0 + g]);
  };
  // winners of an item: CSR slots / generated positions -> positions (the CTA's last warps)
  auto winners_out = [&](int row, int lo, int hi, const int* s_win) {
    int32_t* pout = a.exp + (int64_t)row * E;
    const int32_t* pm = mrow_of(row);
    for (int i = lo + (kTpThreads - 1 - tid); i < hi; i += kTpThreads) {
      const int e = s_win[i];
      pout[i] = e >= 0 ? pm[e] : -e - 1;
    }
  };
  auto bail = [&](int pending_parity) {  // a staged row did not arrive in time: report, let copies land, leave
    if (tid == 0) {
      if (a.status != nullptr) atomicExch(a.status, 4);
      if (pending_parity >= 0) mbar_wait(bar, (uint32_t)pending_parity);
    }
  };
  // ---- prologue: the first item's score row, metadata of the first two items, keys of the first
  if (tid == 0) {
    mbar_init(bar);
    s_next[0] = s_next[1] = 0;
    s_kc[0] = s_kc[1] = 0;
    if (nbytes) bulk_load(s_spill, a.scores + (int64_t)(blockIdx.x / parts) * a.sw, nbytes, bar);
  }
  ts_load_meta(a, meta(0), blockIdx.x / parts, tid, kTpThreads);
  if ((int)blockIdx.x + G < W) ts_load_meta(a, meta(1), ((int)blockIdx.x + G) / parts, tid, kTpThreads);
  __syncthreads();
  if (warp == 0) ts_prefix(meta(0), C, lane);
  bool fail = !(nbytes == 0 || mbar_wait(bar, 0u));
  if (!fail) key_item(blockIdx.x, s_key0, &s_kc[0], meta(0));
  if (__syncthreads_or(fail)) {
    bail(nbytes ? 0 : -1);
    return;
  }
  int it = 0, prev_r = -1, prev_lo = 0, prev_hi = 0;
  for (int wi = blockIdx.x; wi < W; wi += G, ++it) {
    const int cur = it & 1;
    const int nwi = wi + G, nnwi = wi + 2 * G;
    const TsMeta m = meta(it % 3), mn = meta((it + 1) % 3), mnn = meta((it + 2) % 3);
    const int r = wi / parts, part = wi - r * parts;
    const int c_lo = part * C / parts, c_hi = (part + 1) * C / parts;
    if (tid == 0) {
      if (nwi < W && nbytes) {  // the score row was keyed before the last barrier: fetch the next item's
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bulk_load(s_spill, a.scores + (int64_t)(nwi / parts) * a.sw, nbytes, bar);
      }
      s_next[cur ^ 1] = 0;  // the next item's cluster counter (its last use was the previous item)
      s_kc[cur] = 0;        // the chunk counter of item i + 2 (its last use keyed this item)
    }
    if (warp == 1 && nwi < W) ts_prefix(mn, C, lane);  // the next item's quota offsets and cluster order
    if (nnwi < W) ts_load_meta(a, mnn, nnwi / parts, tid, kTpThreads);  // that set last served item i - 1
    if (prev_r >= 0) winners_out(prev_r, prev_lo, prev_hi, s_win0 + (cur ^ 1) * E);
    int32_t* out = a.exp + (int64_t)r * E;
    if (part == 0)
      for (int i = m.base[C] + (kTpThreads - 1 - tid); i < E; i += kTpThreads) out[i] = -1;
    // ---- this item's clusters
    const int32_t* mrow = mrow_of(r);
    const int mo = mo_of(mrow);
    const int gbase = (mo + max(n0, m.cs[c_hi - 1] + m.cl[c_hi - 1]) + 3) & ~3;  // generated keys, as keyed
    const int gcnt = max(0, min(nsp - n0, key_cap - gbase));
    uint16_t* kcur = s_key0 + cur * key_cap;
    const TsRow w{kcur + mo, kcur + gbase, a.scores + (int64_t)r * a.sw, mrow, n0, nsp, gcnt, mo};
    auto key_next = [&]() {
      if (nwi < W) {
        if (nbytes != 0 && !mbar_wait(bar, (uint32_t)((it + 1) & 1))) fail = true;
        else key_item(nwi, s_key0 + (cur ^ 1) * key_cap, &s_kc[cur ^ 1], mn);
      }
    };
    const bool keys_first = warp >= kTpWarps - kTpKeyFirst;
    if (keys_first) key_next();
    ts_select(a, w, m, r, c_lo, c_hi, n, n0, &s_next[cur], s_win0 + cur * E, s_hist[warp], lane);
    if (!keys_first) key_next();
    if (__syncthreads_or(fail)) {
      bail(nwi < W && nbytes ? (it + 1) & 1 : -1);
      return;
    }
    prev_r = r;
    prev_lo = min(m.base[c_lo], E);
    prev_hi = min(m.base[c_hi], E);
  }
  if (prev_r >= 0) winners_out(prev_r, prev_lo, prev_hi, s_win0 + ((it - 1) & 1) * E);
}

// ------------------------------------------------------------------------ top-q, long rows
// For rows whose score row does not fit shared memory (beyond about 47K positions) top-q runs in two
// kernels over a caller workspace of R x ckw 16-bit keys:
//   topq_permute_kernel: one CTA per row stages the score row in chunks of kPmChunk positions (bulk
//     copies; 64 KB chunks let two CTAs share an SM, one staging while the other walks); for each chunk, warps take clusters and key the run of the cluster's members whose
//     positions fall in the chunk (member lists are ascending within a cluster, so each run starts
//     where the previous chunk's ended), writing the keys into the workspace in CSR order; the
//     member list is read once;
//   topq_ck_kernel: one CTA per row (both kernels split a row's clusters over up to four CTAs when
//     there are fewer rows than SMs); warps take the clusters with q > 0 and select from the
//     cluster's contiguous keys in the workspace (register path as topq_stream_kernel, radix path
//     for larger clusters), with generated tokens keyed from the score row.
constexpr int kPmThreads = 1024;
constexpr int kPmChunk = 32768;  // positions staged per pass (64 KB: two CTAs per SM)
constexpr int kPmU = 8;            // 32-member groups a warp loads at once
constexpr int kCkThreads = 256;
constexpr int kCkWarps = kCkThreads / 32;
constexpr int kCkWin = 4096;  // member keys a warp stages in shared memory per window
constexpr int kCkWinSlots = kCkWin + 16 + 64;  // + alignment slack of the 16-byte loads + 64 generated keys

// parts > 1: CTA (row, p) stages every chunk of its row but keys only the clusters [p C / parts, (p+1) C / parts).
__global__ void __launch_bounds__(kPmThreads) topq_permute_kernel(const TopqArgs a, uint16_t* ck, int64_t ckw,
                                                                  int parts) {
  extern __shared__ __align__(128) uint16_t pm_spill[];  // kPmChunk positions
  __shared__ int s_lo[kMaxC];  // per cluster: its first member not keyed yet
  __shared__ int s_next;
  __shared__ __align__(8) uint64_t mbar;
  const int r = blockIdx.x / parts, part = blockIdx.x - r * parts, tid = threadIdx.x, lane = tid & 31;
  const int C = a.C;
  const int c_lo = part * C / parts, c_hi = (part + 1) * C / parts;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  const int npos = min(min(n, n0), a.Lmax);  // member lists hold positions < n0
  const int64_t rC = (int64_t)r * C;
  const uint16_t* sr = a.scores + (int64_t)r * a.sw;
  const int32_t* mrow = a.mem + (int64_t)r * a.Lmax;
  uint16_t* ckr = ck + (int64_t)r * ckw;
  const uint32_t bar = smem_u32(&mbar);
  for (int c = tid; c < C; c += kPmThreads) s_lo[c] = 0;
  if (tid == 0) {
    s_next = c_lo;
    mbar_init(bar);
  }
  __syncthreads();
  int it = 0;
  for (int P0 = 0; P0 < npos; P0 += kPmChunk, ++it) {
    const int P1 = min(npos, P0 + kPmChunk);
    const uint32_t nbytes = (uint32_t)(((P1 - P0) + 7) & ~7) * 2u;
    if (tid == 0) {
      if (it > 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bulk_load(pm_spill, sr + P0, nbytes, bar);
    }
    const bool ok = mbar_wait(bar, (uint32_t)(it & 1));
    if (!__syncthreads_and(ok)) {
      if (tid == 0 && a.status != nullptr) atomicExch(a.status, 4);
      if (!ok) mbar_wait(bar, (uint32_t)(it & 1));
      return;
    }
    // A cluster's members are in ascending position order, so its members inside [P0, P1) are the
    // run that starts at s_lo[c]: warps take clusters and walk their runs kPmU x 32 members at a time.
    while (true) {
      int c = 0;
      if (lane == 0) c = atomicAdd(&s_next, 1);
      c = __shfl_sync(0xffffffffu, c, 0);
      if (c >= c_hi) break;
      const int cs = a.cstart[rC + c], nmem = a.clen[rC + c];
      int lo = s_lo[c];
      while (lo < nmem) {
        int t[kPmU];
#pragma unroll
        for (int u = 0; u < kPmU; ++u) {
          const int i = lo + 32 * u + lane;
          t[u] = i < nmem ? __ldg(mrow + cs + i) : 0x7fffffff;
        }
        int taken = 0;
#pragma unroll
        for (int u = 0; u < kPmU; ++u) {
          // the run starts at the first position >= P0; the lower bound is checked all the same
          const bool in = (unsigned)(t[u] - P0) < (unsigned)(P1 - P0);
          if (in) ckr[cs + lo + 32 * u + lane] = (uint16_t)ukey16(pm_spill[t[u] - P0]);
          taken += __popc(__ballot_sync(0xffffffffu, in));
        }
        lo += taken;
        if (taken < 32 * kPmU) break;
      }
      if (lane == 0) s_lo[c] = lo;
    }
    __syncthreads();  // the staging buffer is refilled by the next pass
    if (tid == 0) s_next = c_lo;
  }
}

// parts > 1 (fewer rows than SMs): CTA (row, p) takes the clusters [p C / parts, (p+1) C / parts) of its row.
__global__ void __launch_bounds__(kCkThreads) topq_ck_kernel(const TopqArgs a, const uint16_t* ck, int64_t ckw,
                                                             int parts) {
  __shared__ int s_base[kMaxC + 1];
  __shared__ int s_q[kMaxC];
  __shared__ int s_next;
  __shared__ int s_win[kCkWarps][32];
  __shared__ int s_hist[kCkWarps][256];
  __shared__ uint64_t s_w64[kCkWarps][64];
  extern __shared__ __align__(16) uint16_t ck_win[];  // per warp kCkWinSlots keys
  const int r = blockIdx.x / parts, part = blockIdx.x - r * parts;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const int C = a.C;
  const int c_lo = part * C / parts, c_hi = (part + 1) * C / parts;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  const int nsp = min(n, a.Lmax);
  const int64_t rC = (int64_t)r * C;
  const uint16_t* ckr = ck + (int64_t)r * ckw;
  const int32_t* mrow = a.mem + (int64_t)r * a.Lmax;
  const int32_t* asg_r = a.asg + (int64_t)r * a.Lmax;
  int32_t* out = a.exp + (int64_t)r * a.E;
  for (int c = tid; c < C; c += kCkThreads) s_q[c] = quota_int(a.quota[rC + c], a.E);
  if (tid == 0) s_next = c_lo;
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      s_base[c] = run;
      run += s_q[c];
    }
    s_base[C] = run;
  }
  __syncthreads();
  if (part == 0)
    for (int i = s_base[C] + tid; i < a.E; i += kCkThreads) out[i] = -1;
  // member keys from the workspace (kb = 0); generated tokens keyed from the score row
  const TsRow w{ckr, nullptr, a.scores + (int64_t)r * a.sw, mrow, n0, nsp, 0, 0};
  int* hist = s_hist[warp];
  uint16_t* wk = ck_win + (size_t)warp * kCkWinSlots;
  while (true) {
    int c = 0;
    if (lane == 0) {
      do {
        c = atomicAdd(&s_next, 1);
      } while (c < c_hi && s_q[c] <= 0);
    }
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= c_hi) break;
    const int q = s_q[c], base = s_base[c];
    const int cs = a.cstart[rC + c], nmem = a.clen[rC + c];
    const int cnt = a.reclist ? a.reccnt[rC + c] : 0x7fffffff;
    const bool use_list = a.reclist != nullptr && cnt <= a.rmax;
    const int32_t* rec = use_list ? a.reclist + (rC + c) * a.rmax : nullptr;
    const int ngen = use_list ? cnt : 0;
    if (use_list && q <= kSmallQ && ngen <= 64 && nmem + 3 <= 1024) {
      const int span = nmem + 3;
      int* win = s_win[warp];
      if (span <= 256)
        topq_keys_regs<8>(w, cs, nmem, rec, ngen, q, win, 32, lane);
      else if (span <= 512)
        topq_keys_regs<16>(w, cs, nmem, rec, ngen, q, win, 32, lane);
      else
        topq_keys_regs<32>(w, cs, nmem, rec, ngen, q, win, 32, lane);
      __syncwarp();
      if (lane < q && base + lane < a.E) {
        const int e = win[lane];
        out[base + lane] = e >= 0 ? mrow[e] : -e - 1;
      }
      __syncwarp();
      continue;
    }
    const int ngen_scan = max(0, n - n0);
    auto pos_of = [&](int idx) -> int {
      if (idx < nmem) return mrow[cs + idx];
      return use_list ? rec[idx - nmem] : n0 + (idx - nmem);
    };
    // a cluster that fits the window is staged once: its member keys with 16-byte loads (all in
    // flight at once), then up to 64 listed generated tokens' keys after them
    const bool staged = nmem <= kCkWin;
    const bool gen_staged = staged && use_list && ngen <= 64;
    const int so = cs & 7;  // wk[so + i] = key of member i
    if (staged) {
      const int nv = (so + nmem + 7) >> 3;  // ends at most at Lmax rounded up to 8 = the row stride
      __syncwarp();
#pragma unroll 4
      for (int j = lane; j < nv; j += 32)
        reinterpret_cast<int4*>(wk)[j] = __ldg(reinterpret_cast<const int4*>(ckr + (cs - so)) + j);
      __syncwarp();
      if (gen_staged)
        for (int j = lane; j < ngen; j += 32) wk[so + nmem + j] = (uint16_t)ts_key_at(w, rec[j]);
      __syncwarp();
    }
    // threshold + sort: the k-th largest lane maximum bounds the answer from below (warp_topk_sorted)
    if (gen_staged && q <= 32) {
      uint64_t srt[2], kth;
      auto word = [&](int i) -> uint64_t {
        return ((uint64_t)wk[so + i] << 32) | (uint64_t)(0xffffffffu - (uint32_t)i);
      };
      if (warp_topk_sorted(nmem + ngen, q, word, s_w64[warp], srt, kth)) {
        // lanes < q hold the winners in key order; each finds its slot by list index (= position order)
        const int idx = (int)(0xffffffffu - (uint32_t)srt[0]);
        int rank = 0;
        for (int j = 0; j < q; ++j) rank += __shfl_sync(0xffffffffu, idx, j) < idx ? 1 : 0;
        if (lane < q && base + rank < a.E) out[base + rank] = pos_of(idx);
        __syncwarp();
        continue;
      }
    }
    // radix path over (list index, key): members' keys, then generated tokens
    auto for_each = [&](auto&& f) {
      if (staged) {
        for (int i0 = 0; i0 < nmem; i0 += 32) {
          const int i = i0 + lane;
          const bool v = i < nmem;
          f(v, i, v ? (uint32_t)wk[so + i] : 0u);
        }
      } else {
        // members in windows of kCkWin keys, each staged with 16-byte loads
        for (int w0 = 0; w0 < nmem; w0 += kCkWin) {
          const int wn = min(kCkWin, nmem - w0);
          const int g0 = cs + w0, a0 = g0 & ~7, o = g0 - a0;
          const int nv = (o + wn + 7) >> 3;
          __syncwarp();
#pragma unroll 4
          for (int j = lane; j < nv; j += 32)
            reinterpret_cast<int4*>(wk)[j] = __ldg(reinterpret_cast<const int4*>(ckr + a0) + j);
          __syncwarp();
          for (int i0 = 0; i0 < wn; i0 += 32) {
            const int i = i0 + lane;
            const bool v = i < wn;
            f(v, w0 + i, v ? (uint32_t)wk[o + i] : 0u);
          }
        }
      }
      if (gen_staged) {
        for (int i0 = 0; i0 < ngen; i0 += 32) {
          const int i = i0 + lane;
          const bool v = i < ngen;
          f(v, nmem + i, v ? (uint32_t)wk[so + nmem + i] : 0u);
        }
      } else if (use_list) {
        for (int i0 = 0; i0 < cnt; i0 += 32) {
          const int i = i0 + lane;
          const bool v = i < cnt;
          f(v, nmem + i, v ? ts_key_at(w, rec[i]) : 0u);
        }
      } else {
        for (int i0 = 0; i0 < ngen_scan; i0 += 32) {
          const int t = n0 + i0 + lane;
          const bool v = (i0 + lane < ngen_scan) && asg_r[t] == c;
          f(v, nmem + i0 + lane, v ? ts_key_at(w, t) : 0u);
        }
      }
    };
    int above = 0, hi = 0, lo = 0;
    bool all = false;
    for (int pass = 0; pass < 2 && !all; ++pass) {
      for (int b = lane; b < 256; b += 32) hist[b] = 0;
      __syncwarp();
      for_each([&](bool v, int, uint32_t k) {
        // lanes with the same bin add once (a cluster's keys share few high bytes)
        const bool part = v && (pass == 0 || (int)(k >> 8) == hi);
        const int bin = part ? (int)(pass == 0 ? (k >> 8) : (k & 255)) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, bin);
        if (part && __ffs(peers) - 1 == lane) atomicAdd(&hist[bin], __popc(peers));
      });
      __syncwarp();
      int cnt8[8], sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt8[i] = hist[255 - 8 * lane - i];
        sum += cnt8[i];
      }
      int incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += x;
      }
      const int excl = incl - sum;
      const int need = q - above;
      int fb = -1, fa = 0;
      if (excl < need && incl >= need) {
        int run = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (fb < 0 && run + cnt8[i] >= need) {
            fb = 255 - 8 * lane - i;
            fa = run;
          }
          run += cnt8[i];
        }
      }
      const unsigned who = __ballot_sync(0xffffffffu, fb >= 0);
      if (who == 0u) {
        all = true;
      } else {
        const int src = __ffs(who) - 1;
        const int d = __shfl_sync(0xffffffffu, fb, src);
        above += __shfl_sync(0xffffffffu, fa, src);
        if (pass == 0) hi = d;
        else lo = d;
      }
      __syncwarp();
    }
    const uint32_t T = all ? 0u : (((uint32_t)hi << 8) | (uint32_t)lo);
    const int need_eq = all ? 0 : q - above;
    int taken = 0, ties = 0;
    for_each([&](bool v, int idx, uint32_t k) {
      const bool gt = v && k > T;
      const bool eq = v && k == T;
      const unsigned beq = __ballot_sync(0xffffffffu, eq);
      const bool take = gt || (eq && ties + __popc(beq & lt) < need_eq);
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      const int slot = taken + __popc(bt & lt);
      if (take && slot < q && base + slot < a.E) out[base + slot] = pos_of(idx);
      taken += __popc(bt);
      ties += __popc(beq);
    });
    __syncwarp();
  }
}

// ------------------------------------------------------------------------ residual proxies (+ flash)
// One CTA (8 warps) per row; warp w owns the clusters c = c0 + w + 8k (k < 8) of each 64-cluster
// chunk and keeps their running sums Sk - sum k, Sv - sum v in registers (lane <-> dims lane + 32i).
// The row's read tokens (sel, then the exp slots) are gathered 32 at a time into a double-buffered
// shared-memory ring (cp.async), so the next chunk loads while this one is used.  For every chunk a
// warp subtracts, in list order, the tokens of its clusters (a cluster's exp tokens are one
// contiguous segment [base_c, base_c + q_c)); with ATTEND the warps also run the online softmax
// over the chunk's tokens (P1/P2).  At the end each warp turns its sums into kbar' / vbar' (bf16, as
// the reference stores them) and ln n', writes them if asked, and with ATTEND attends them as
// proxies (P3) straight from registers; the 8 warp states are merged into the output.
constexpr int kRW = 8;         // warps per CTA
constexpr int kRPer = 8;       // clusters per warp per chunk
constexpr int kChunkC = kRW * kRPer;
constexpr int kTok = 32;       // tokens per gather buffer
constexpr int kMaxRead = 2048;  // NS + E

struct ResidArgs {
  const __nv_bfloat16* q;  // ATTEND only
  int64_t q_stride;
  const __nv_bfloat16* K;
  const __nv_bfloat16* V;
  int Lmax, C, NS, E;
  const int32_t* asg;
  const int32_t* sel;
  const int32_t* exp;
  const float* Sk;
  const float* Sv;
  const float* nt;
  const float* quota;
  const float* zdot;    // may be null; proxy_flash_kernel then reads Sk
  __nv_bfloat16* kbar;  // may be null (then not written)
  __nv_bfloat16* vbar;
  float* logn;
  void* out;  // ATTEND only
  int64_t out_stride;
  int out_f32;
  float qk_scale;  // sm_scale * log2(e)
  int32_t* status;
};

struct SoftmaxState {
  float m, l, acc[4];
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    l = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0.f;
  }
  // one entry with log2-domain logit z (warp-uniform) and value lanes v[4]
  __device__ __forceinline__ void add(float z, const float (&v)[4]) {
    if (z == -INFINITY) return;
    const float mx = fmaxf(m, z);
    const float alpha = exp2f(m - mx);
    const float p = exp2f(z - mx);
    l = fmaf(l, alpha, p);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = fmaf(acc[i], alpha, p * v[i]);
    m = mx;
  }
};

__device__ __forceinline__ float warp_dot4(const float (&a)[4], const float (&b)[4]) {
  float d = a[0] * b[0];
  d = fmaf(a[1], b[1], d);
  d = fmaf(a[2], b[2], d);
  d = fmaf(a[3], b[3], d);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
  return d;
}

template <bool ATTEND>
__global__ void __launch_bounds__(kRW * 32, 2) residual_kernel(const ResidArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kv = r / kG;
  const int C = a.C;
  __shared__ __align__(16) __nv_bfloat16 sK[2][kTok][kD];
  __shared__ __align__(16) __nv_bfloat16 sV[2][kTok][kD];
  __shared__ int s_tok[kMaxRead];
  __shared__ int16_t s_tc[kMaxRead];
  __shared__ int s_base[kMaxC + 1];
  __shared__ int s_q[kMaxC];
  __shared__ float s_m[kRW], s_l[kRW];
  for (int c = tid; c < C; c += blockDim.x) s_q[c] = quota_int(a.quota[(int64_t)r * C + c], a.E);
  const int NT = a.NS + a.E;
  for (int j = tid; j < NT; j += blockDim.x) {
    const int t = j < a.NS ? a.sel[(int64_t)r * a.NS + j] : a.exp[(int64_t)r * a.E + (j - a.NS)];
    const bool v = t >= 0 && t < a.Lmax;
    s_tok[j] = v ? t : -1;
    s_tc[j] = v ? (int16_t)a.asg[(int64_t)r * a.Lmax + t] : (int16_t)-1;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      s_base[c] = run;
      run += s_q[c];
    }
    s_base[C] = run;
  }
  float qv[4];
  SoftmaxState sm;
  sm.init();
  if (ATTEND) {
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = __bfloat162float(a.q[(int64_t)r * a.q_stride + lane + 32 * i]);
  }
  const __nv_bfloat16* Kr = a.K + (int64_t)kv * a.Lmax * kD;
  const __nv_bfloat16* Vr = a.V + (int64_t)kv * a.Lmax * kD;
  const int nchunks = (NT + kTok - 1) / kTok;
  __syncthreads();
  for (int c0 = 0; c0 < C; c0 += kChunkC) {
    const bool first = c0 == 0;  // the token streams are attended during the first cluster chunk
    // this warp's clusters and their running sums
    float sk[kRPer][4], sv[kRPer][4];
#pragma unroll
    for (int k = 0; k < kRPer; ++k) {
      const int c = c0 + warp + kRW * k;
      const int64_t base = ((int64_t)r * C + min(c, C - 1)) * kD;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sk[k][i] = c < C ? a.Sk[base + lane + 32 * i] : 0.f;
        sv[k][i] = c < C ? a.Sv[base + lane + 32 * i] : 0.f;
      }
    }
    auto gather = [&](int ch) {  // rows of chunk ch into buffer ch & 1 (one cp.async group)
      const int j0 = ch * kTok, nj = min(kTok, NT - j0), b = ch & 1;
      for (int e = tid; e < nj * 32; e += blockDim.x) {
        const int j = e >> 5, part = e & 31;  // part < 16: K row, else V row
        const int t = s_tok[j0 + j];
        const int tc = s_tc[j0 + j];
        if (t >= 0 && (first || (tc >= c0 && tc < c0 + kChunkC))) {
          const __nv_bfloat16* src = (part < 16 ? Kr : Vr) + (int64_t)t * kD + (part & 15) * 8;
          __nv_bfloat16* dst = (part < 16 ? &sK[b][j][0] : &sV[b][j][0]) + (part & 15) * 8;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    gather(0);
    for (int ch = 0; ch < nchunks; ++ch) {
      if (ch + 1 < nchunks) {
        gather(ch + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      __syncthreads();
      const int j0 = ch * kTok, nj = min(kTok, NT - j0), b = ch & 1;
      // residual: this warp's clusters, tokens in list order
#pragma unroll
      for (int k = 0; k < kRPer; ++k) {
        const int c = c0 + warp + kRW * k;
        if (c >= C) break;
        auto sub = [&](int j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            sk[k][i] = __fsub_rn(sk[k][i], __bfloat162float(sK[b][j][lane + 32 * i]));
            sv[k][i] = __fsub_rn(sv[k][i], __bfloat162float(sV[b][j][lane + 32 * i]));
          }
        };
        for (int j = j0; j < min(j0 + nj, a.NS); ++j)
          if (s_tc[j] == c) sub(j - j0);
        const int e_lo = max(j0, a.NS + s_base[c]), e_hi = min(j0 + nj, a.NS + min(s_base[c + 1], a.E));
        for (int j = e_lo; j < e_hi; ++j)
          if (s_tok[j] >= 0) sub(j - j0);
      }
      if (ATTEND && first) {  // P1/P2: warp w takes the chunk's tokens w, w+8, ...
        for (int j = warp; j < nj; j += kRW) {
          if (s_tok[j0 + j] < 0) continue;
          float kx[4], vx[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kx[i] = __bfloat162float(sK[b][j][lane + 32 * i]);
            vx[i] = __bfloat162float(sV[b][j][lane + 32 * i]);
          }
          sm.add(warp_dot4(qv, kx) * a.qk_scale, vx);
        }
      }
      __syncthreads();  // buffer b is refilled by chunk ch + 2
    }
    // proxies of this warp's clusters
#pragma unroll
    for (int k = 0; k < kRPer; ++k) {
      const int c = c0 + warp + kRW * k;
      if (c >= C) break;
      const float nr = __fsub_rn(a.nt[(int64_t)r * C + c], a.quota[(int64_t)r * C + c]);
      const float inv = __fdiv_rn(1.f, fmaxf(nr, 1.f));
      const int64_t base = ((int64_t)r * C + c) * kD;
      float kb[4], vb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat16 kh = __float2bfloat16_rn(__fmul_rn(sk[k][i], inv));
        const __nv_bfloat16 vh = __float2bfloat16_rn(__fmul_rn(sv[k][i], inv));
        kb[i] = __bfloat162float(kh);
        vb[i] = __bfloat162float(vh);
        if (a.kbar != nullptr) {
          a.kbar[base + lane + 32 * i] = kh;
          a.vbar[base + lane + 32 * i] = vh;
        }
      }
      float ln = 0.f;
      if (lane == 0) {
        ln = nr > 0.5f ? ln_f(fmaxf(nr, 1.f)) : -INFINITY;
        if (a.logn != nullptr) a.logn[(int64_t)r * C + c] = ln;
      }
      if (ATTEND) {
        ln = __shfl_sync(0xffffffffu, ln, 0);
        if (ln > -INFINITY) sm.add(fmaf(warp_dot4(qv, kb), a.qk_scale, ln * kLog2e), vb);
      }
    }
  }
  if (!ATTEND) return;
  // the gather ring is free now (every chunk loop ended with a barrier): merge area for the warps
  float(*s_acc)[kD] = reinterpret_cast<float(*)[kD]>(&sK[0][0][0]);
  if (lane == 0) {
    s_m[warp] = sm.m;
    s_l[warp] = sm.l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s_acc[warp][lane + 32 * i] = sm.acc[i];
  __syncthreads();
  if (tid < kD) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kRW; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f, A = 0.f;
    if (M > -INFINITY) {
#pragma unroll
      for (int w = 0; w < kRW; ++w) {
        const float wt = exp2f(s_m[w] - M);
        L = fmaf(wt, s_l[w], L);
        A = fmaf(wt, s_acc[w][tid], A);
      }
    }
    const float o = L > 0.f ? A / L : 0.f;
    if (a.out_f32)
      reinterpret_cast<float*>(a.out)[(int64_t)r * a.out_stride + tid] = o;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)r * a.out_stride + tid] = __float2bfloat16_rn(o);
  }
}


// ------------------------------------------------------------------------------------------------
// Residual proxies folded into the flash pass (no proxy tensors kept).  For a live cluster c
// (n'_c = nt_c - q_c > 0.5) with read set R_c (its selected and expanded tokens):
//   q.kbar'_c = (q.Sk_c - sum_{t in R_c} q.k_t) / max(n'_c, 1)
// so the proxy logit needs only the SCALAR q.dk_c, a sum of the token dots the flash computes
// anyway; and with w_c = p_c / max(n'_c, 1) the value side is
//   sum_t p_t v_t + sum_c p_c vbar'_c = sum_t (p_t - w_c(t)) v_t + sum_c w_c Sv_c.
// Pass A gathers K rows and Sk rows (token and proxy logits), pass B gathers V rows and Sv rows
// with the final weights.  No per-cluster vector sums are held, so a CTA is 4 warps with a few KB
// of shared memory and every load of a pass can be in flight at once.  The proxies are the fp32
// estimator's (kbar' = (Sk - dk)/n' unrounded); the bf16-rounded proxies of the reference's
// _k_resid_norm (ours_fused.py:388-407) are produced by residual_kernel when they are requested.
constexpr int kPF = 128;      // threads per CTA
constexpr int kPFHalf = kPF / 16;
constexpr int kPFU = 8;       // rows a half-warp has in flight

struct PFShared {
  int* tok;      // [NT] token position or -1
  int16_t* cl;   // [NT] cluster of the token or -1
  float* z;      // [NT] q.k dot, then the pass-B coefficient
  int* base;     // [C + 1] exclusive prefix of the quotas
  float* qsk;    // [C] q.Sk_c (live clusters)
  float* w;      // [C] proxy weight / max(n', 1), 0 when not live
  float* zc;     // [C] proxy logit (log2 domain) or -inf
  float* inv;    // [C]
};

__device__ __forceinline__ float hw_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x;
}

__device__ __forceinline__ float dot8(const float* q, const uint4& w) {
  float d = q[0] * bf_lo(w.x);
  d = fmaf(q[1], bf_hi(w.x), d);
  d = fmaf(q[2], bf_lo(w.y), d);
  d = fmaf(q[3], bf_hi(w.y), d);
  d = fmaf(q[4], bf_lo(w.z), d);
  d = fmaf(q[5], bf_hi(w.z), d);
  d = fmaf(q[6], bf_lo(w.w), d);
  d = fmaf(q[7], bf_hi(w.w), d);
  return d;
}

__device__ __forceinline__ float dot8f(const float* q, const float4& a, const float4& b) {
  float d = q[0] * a.x;
  d = fmaf(q[1], a.y, d);
  d = fmaf(q[2], a.z, d);
  d = fmaf(q[3], a.w, d);
  d = fmaf(q[4], b.x, d);
  d = fmaf(q[5], b.y, d);
  d = fmaf(q[6], b.z, d);
  d = fmaf(q[7], b.w, d);
  return d;
}

__device__ __forceinline__ float block_reduce_pf(float v, bool is_max, float* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, off);
    v = is_max ? fmaxf(v, o) : v + o;
  }
  __syncthreads();
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  float r = s_red[0];
#pragma unroll
  for (int i = 1; i < kPF / 32; ++i) r = is_max ? fmaxf(r, s_red[i]) : r + s_red[i];
  return r;
}

// NCTA > 1 (few rows): a row is spread over a cluster of NCTA CTAs.  CTA k makes the token dots of
// its share of the read list (and the q.Sk dots of its share of the clusters); the CTAs exchange them
// through distributed shared memory, each then forms the same proxy logits, normaliser and
// coefficients, and gathers its share of the V / Sv rows; rank 0 adds the NCTA partial outputs in
// rank order.  Token dots, proxies and softmax statistics are those of NCTA = 1 bit for bit; the
// output differs only by the order of that last sum.
template <int NCTA>
__global__ void __launch_bounds__(kPF, 8) proxy_flash_kernel(const ResidArgs a) {
  extern __shared__ __align__(16) unsigned char pf_smem[];
  namespace cg = cooperative_groups;
  const int r = blockIdx.x / NCTA;
  const int rank = NCTA > 1 ? (int)cg::this_cluster().block_rank() : 0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hw = tid >> 4, hl = tid & 15;
  const int kv = r / kG;
  const int C = a.C, NS = a.NS, NT = a.NS + a.E;
  // this CTA's share of the read list and of the clusters
  const int j_lo = rank * NT / NCTA, j_hi = (rank + 1) * NT / NCTA;
  const int c_lo = rank * C / NCTA, c_hi = (rank + 1) * C / NCTA;
  __shared__ float s_red[kPF / 32];
  __shared__ __align__(16) float s_acc[kPFHalf][kD];
  PFShared S;
  {
    unsigned char* p = pf_smem;
    S.z = reinterpret_cast<float*>(p);
    p += sizeof(float) * ((NT + 3) & ~3);
    S.qsk = reinterpret_cast<float*>(p);
    p += sizeof(float) * ((C + 3) & ~3);
    S.w = reinterpret_cast<float*>(p);
    p += sizeof(float) * ((C + 3) & ~3);
    S.zc = reinterpret_cast<float*>(p);
    p += sizeof(float) * ((C + 3) & ~3);
    S.inv = reinterpret_cast<float*>(p);
    p += sizeof(float) * ((C + 3) & ~3);
    S.tok = reinterpret_cast<int*>(p);
    p += sizeof(int) * ((NT + 3) & ~3);
    S.base = reinterpret_cast<int*>(p);
    p += sizeof(int) * ((C + 4) & ~3);
    S.cl = reinterpret_cast<int16_t*>(p);
  }
  const int64_t rowC = (int64_t)r * C;
  // ---- row metadata: quotas (prefix), tokens, clusters of the selected tokens
  for (int c = tid; c < C; c += kPF) S.w[c] = a.quota[rowC + c];  // staged quota (w is free until later)
  for (int j = tid; j < NT; j += kPF) {
    const int t = j < NS ? a.sel[(int64_t)r * NS + j] : a.exp[(int64_t)r * a.E + (j - NS)];
    const bool v = t >= 0 && t < a.Lmax;
    S.tok[j] = v ? t : -1;
    if (j < NS) {  // an assignment outside [0, C) counts as none
      const int ca = v ? a.asg[(int64_t)r * a.Lmax + t] : -1;
      S.cl[j] = (int16_t)(ca >= 0 && ca < C ? ca : -1);
    }
  }
  float qv[8];
  {
    const uint4 qw = *reinterpret_cast<const uint4*>(a.q + (int64_t)r * a.q_stride + hl * 8);
    qv[0] = bf_lo(qw.x); qv[1] = bf_hi(qw.x); qv[2] = bf_lo(qw.y); qv[3] = bf_hi(qw.y);
    qv[4] = bf_lo(qw.z); qv[5] = bf_hi(qw.z); qv[6] = bf_lo(qw.w); qv[7] = bf_hi(qw.w);
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefix of the quotas, lanes own consecutive runs of clusters
    const int per = (C + 31) / 32;
    const int c0 = lane * per, c1 = min(C, c0 + per);
    int run = 0;
    for (int c = c0; c < c1; ++c) run += quota_int(S.w[c], a.E);
    int incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int ex = incl - run;
    for (int c = c0; c < c1; ++c) {
      S.base[c] = ex;
      ex += quota_int(S.w[c], a.E);
    }
    if (lane == 31) S.base[C] = incl;
  }
  __syncthreads();
  for (int j = NS + tid; j < NT; j += kPF) {  // expanded slot -> its cluster segment
    const int slot = j - NS;
    int c = -1;
    if (S.tok[j] >= 0 && slot < S.base[C]) {
      int lo = 0, hi = C;  // largest c with base[c] <= slot
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (S.base[mid] <= slot) lo = mid; else hi = mid;
      }
      c = lo;
    }
    S.cl[j] = (int16_t)c;
  }
  for (int c = tid; c < C; c += kPF) {
    const float nr = __fsub_rn(a.nt[rowC + c], S.w[c]);
    S.inv[c] = nr > 0.5f ? __fdiv_rn(1.f, fmaxf(nr, 1.f)) : 0.f;
    // log2 n' (the output is held to the estimator's tolerance, not to the proxies' bits)
    S.zc[c] = nr > 0.5f ? __log2f(fmaxf(nr, 1.f)) : -INFINITY;  // completed below
  }
  __syncthreads();
  const __nv_bfloat16* Kr = a.K + (int64_t)kv * a.Lmax * kD + hl * 8;
  const __nv_bfloat16* Vr = a.V + (int64_t)kv * a.Lmax * kD + hl * 8;
  // ---- pass A: token dots (K rows) and q.Sk for live clusters.  The loops that reduce over a
  //      half-warp with full-mask shuffles run a CTA-uniform trip count: with the half-warp index in
  //      the loop bound, the two halves of a warp would differ by one trip whenever NT = 2w + 1 (mod
  //      64), and one half would shuffle with lanes that have left the loop.
  for (int jb = j_lo; jb < j_hi; jb += kPFHalf * kPFU) {
    uint4 kw[kPFU];
#pragma unroll
    for (int u = 0; u < kPFU; ++u) {
      const int j = jb + hw + u * kPFHalf;
      const int t = j < j_hi ? S.tok[j] : -1;
      kw[u] = t >= 0 ? ldg_stream(reinterpret_cast<const uint4*>(Kr + (int64_t)t * kD)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kPFU; ++u) {
      const int j = jb + hw + u * kPFHalf;
      const float d = hw_sum(dot8(qv, kw[u]));
      if (hl == 0 && j < j_hi) S.z[j] = d;
    }
  }
  const float* Skr = a.Sk + rowC * kD + hl * 8;
  if (a.zdot != nullptr) {
    // q . (Sk_b - selected tokens) = zdot_b * n_t(b): the tail mean's dot from the ErrorGate pass
    for (int c = tid; c < C; c += kPF)
      if (S.inv[c] > 0.f) S.qsk[c] = __fmul_rn(a.zdot[rowC + c], a.nt[rowC + c]);
  }
  for (int cb = c_lo; a.zdot == nullptr && cb < c_hi; cb += kPFHalf * 4) {
    float4 x[4], y[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = cb + hw + u * kPFHalf;
      const bool live = c < c_hi && S.inv[c] > 0.f;
      x[u] = live ? __ldg(reinterpret_cast<const float4*>(Skr + (int64_t)c * kD)) : make_float4(0.f, 0.f, 0.f, 0.f);
      y[u] = live ? __ldg(reinterpret_cast<const float4*>(Skr + (int64_t)c * kD + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = cb + hw + u * kPFHalf;
      const float d = hw_sum(dot8f(qv, x[u], y[u]));
      if (hl == 0 && c < c_hi) S.qsk[c] = d;
    }
  }
  if constexpr (NCTA > 1) {  // every CTA gets the other CTAs' token dots (and q.Sk dots)
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    for (int k = 0; k < NCTA; ++k) {
      if (k == rank) continue;
      const float* rz = cluster.map_shared_rank(S.z, k);
      for (int j = k * NT / NCTA + tid; j < (k + 1) * NT / NCTA; j += kPF) S.z[j] = rz[j];
      if (a.zdot == nullptr) {
        const float* rq = cluster.map_shared_rank(S.qsk, k);
        for (int c = k * C / NCTA + tid; c < (k + 1) * C / NCTA; c += kPF) S.qsk[c] = rq[c];
      }
    }
    cluster.sync();  // no CTA overwrites its dots (with coefficients, below) while a peer still reads them
  }
  __syncthreads();
  // ---- proxy logits: one thread per cluster sums q.dk_c over the cluster's read tokens in a fixed
  //      order (selected tokens in list order, then its slot segment)
  for (int c = tid; c < C; c += kPF) {
    if (!(S.inv[c] > 0.f)) continue;
    float part = 0.f;
    if (a.zdot == nullptr)  // with zdot the selected tokens are already out of the tail mean
      for (int j = 0; j < NS; ++j)
        if (S.cl[j] == c) part += S.z[j];
    const int e0 = NS + S.base[c], e1 = NS + min(S.base[c + 1], a.E);
    for (int j = e0; j < e1; ++j)
      if (S.tok[j] >= 0) part += S.z[j];
    S.zc[c] = fmaf(__fmul_rn(__fsub_rn(S.qsk[c], part), S.inv[c]), a.qk_scale, S.zc[c]);
  }
  __syncthreads();
  // ---- softmax normaliser: max over token and proxy logits, then weights
  float mx = -INFINITY;
  for (int j = tid; j < NT; j += kPF)
    if (S.tok[j] >= 0) mx = fmaxf(mx, S.z[j] * a.qk_scale);
  for (int c = tid; c < C; c += kPF) mx = fmaxf(mx, S.zc[c]);
  const float M = block_reduce_pf(mx, true, s_red);
  float lsum = 0.f;
  for (int c = tid; c < C; c += kPF) {
    const float p = S.zc[c] > -INFINITY ? exp2f(S.zc[c] - M) : 0.f;
    lsum += p;
    S.w[c] = __fmul_rn(p, S.inv[c]);
  }
  __syncthreads();  // w complete before the token coefficients read it
  for (int j = tid; j < NT; j += kPF) {
    float coef = 0.f;
    if (S.tok[j] >= 0) {
      const float p = exp2f(S.z[j] * a.qk_scale - M);
      lsum += p;
      const int c = S.cl[j];
      coef = c >= 0 ? __fsub_rn(p, S.w[c]) : p;
    }
    S.z[j] = coef;
  }
  const float L = block_reduce_pf(lsum, false, s_red);  // its barriers also publish z and w
  // ---- pass B: V rows with the coefficients, Sv rows with the proxy weights
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j0 = j_lo + hw; j0 < j_hi; j0 += kPFHalf * kPFU) {
    uint4 vw[kPFU];
#pragma unroll
    for (int u = 0; u < kPFU; ++u) {
      const int j = j0 + u * kPFHalf;
      const int t = j < j_hi ? S.tok[j] : -1;
      vw[u] = t >= 0 ? ldg_stream(reinterpret_cast<const uint4*>(Vr + (int64_t)t * kD)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kPFU; ++u) {
      const int j = j0 + u * kPFHalf;
      const float cf = j < j_hi ? S.z[j] : 0.f;
      acc[0] = fmaf(cf, bf_lo(vw[u].x), acc[0]);
      acc[1] = fmaf(cf, bf_hi(vw[u].x), acc[1]);
      acc[2] = fmaf(cf, bf_lo(vw[u].y), acc[2]);
      acc[3] = fmaf(cf, bf_hi(vw[u].y), acc[3]);
      acc[4] = fmaf(cf, bf_lo(vw[u].z), acc[4]);
      acc[5] = fmaf(cf, bf_hi(vw[u].z), acc[5]);
      acc[6] = fmaf(cf, bf_lo(vw[u].w), acc[6]);
      acc[7] = fmaf(cf, bf_hi(vw[u].w), acc[7]);
    }
  }
  const float* Svr = a.Sv + rowC * kD + hl * 8;
  for (int c0 = c_lo + hw; c0 < c_hi; c0 += kPFHalf * 4) {
    float4 x[4], y[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * kPFHalf;
      const bool use = c < c_hi && S.w[c] != 0.f;
      x[u] = use ? __ldg(reinterpret_cast<const float4*>(Svr + (int64_t)c * kD)) : make_float4(0.f, 0.f, 0.f, 0.f);
      y[u] = use ? __ldg(reinterpret_cast<const float4*>(Svr + (int64_t)c * kD + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * kPFHalf;
      const float wc = c < c_hi ? S.w[c] : 0.f;
      acc[0] = fmaf(wc, x[u].x, acc[0]);
      acc[1] = fmaf(wc, x[u].y, acc[1]);
      acc[2] = fmaf(wc, x[u].z, acc[2]);
      acc[3] = fmaf(wc, x[u].w, acc[3]);
      acc[4] = fmaf(wc, y[u].x, acc[4]);
      acc[5] = fmaf(wc, y[u].y, acc[5]);
      acc[6] = fmaf(wc, y[u].z, acc[6]);
      acc[7] = fmaf(wc, y[u].w, acc[7]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) s_acc[hw][hl * 8 + i] = acc[i];
  __syncthreads();
  float A = 0.f;
  if (tid < kD) {
#pragma unroll
    for (int h = 0; h < kPFHalf; ++h) A += s_acc[h][tid];
  }
  if constexpr (NCTA > 1) {  // rank 0 adds the partial outputs in rank order
    cg::cluster_group cluster = cg::this_cluster();
    if (tid < kD) s_acc[0][tid] = A;  // a thread rewrites only the column it has summed
    cluster.sync();
    A = 0.f;
    if (rank == 0 && tid < kD)
      for (int k = 0; k < NCTA; ++k) A += cluster.map_shared_rank(&s_acc[0][0], k)[tid];
    cluster.sync();  // every CTA stays until rank 0 has read its partial output
    if (rank != 0) return;
  }
  if (tid < kD) {
    const float o = L > 0.f ? A / L : 0.f;
    if (a.out_f32)
      reinterpret_cast<float*>(a.out)[(int64_t)r * a.out_stride + tid] = o;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)r * a.out_stride + tid] = __float2bfloat16_rn(o);
  }
}

size_t proxy_flash_smem(int NT, int C) {
  return sizeof(float) * ((NT + 3) & ~3) + 4 * sizeof(float) * ((C + 3) & ~3) + sizeof(int) * ((NT + 3) & ~3) +
         sizeof(int) * ((C + 4) & ~3) + sizeof(int16_t) * ((NT + 7) & ~7);
}

}  // namespace
}  // namespace oa

using namespace oa;

extern "C" int oa_errorgate_waterfill(const void* q, int64_t q_stride, const void* K, int64_t B, int64_t hkv,
                                      int64_t Lmax, int64_t C, const int32_t* asg, const int32_t* sel, int64_t n_sel,
                                      const float* Sk, const float* Sk2, const float* nb, float E, float* score,
                                      float* nt, float* quota, float* zdot, int32_t* status, void* stream) {
  const char* fn = "oa_errorgate_waterfill";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= kMaxC, "%s: need 0 < C <= %d (C=%lld)", fn, kMaxC, (long long)C);
  OA_REQUIRE_HKV(fn, hkv);
  const int64_t R = B * kG * hkv;
  OA_REQUIRE(n_sel > 0 && n_sel <= 512, "%s: n_sel=%lld outside [1, 512]", fn, (long long)n_sel);
  OA_REQUIRE(q && K && asg && sel && Sk && Sk2 && nb && score && nt && quota, "%s: null pointer", fn);
  OA_REQUIRE(E >= 0.f, "%s: negative budget", fn);
  OA_REQUIRE(oa_aligned16(Sk) && oa_aligned16(Sk2), "%s: Sk / Sk2 must be 16-byte aligned", fn);
  GateArgs a{static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<const __nv_bfloat16*>(K), (int)Lmax, (int)C,
             (int)n_sel, asg, sel, Sk, Sk2, nb, E, score, nt, quota, zdot, status};
  const size_t smem = eg_smem_bytes((int)C, (int)n_sel);
  // few rows (small batches): 8 warps per row shorten each row's chain; a full batch keeps 2 warps per
  // row so that every row is resident at once.  Results do not depend on the choice.
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (R <= 2 * sms) {
    if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(errorgate_waterfill_kernel<256>), smem, fn)) return rc;
    errorgate_waterfill_kernel<256><<<(unsigned)R, 256, smem, static_cast<cudaStream_t>(stream)>>>(a);
  } else {
    if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(errorgate_waterfill_kernel<kEgThreads>), smem, fn))
      return rc;
    errorgate_waterfill_kernel<kEgThreads><<<(unsigned)R, kEgThreads, smem, static_cast<cudaStream_t>(stream)>>>(a);
  }
  return oa_check_launch(fn);
}

namespace oa {
namespace {
size_t ts_smem_bytes(int64_t Lmax, int64_t E) {  // shared memory of topq_stream_kernel for one row
  const size_t spill_bytes = (size_t)((Lmax + 7) & ~7ll) * 2;
  const int key_cap = (int)(((Lmax + 7) & ~7ll) + 1040);  // list slack of the register path
  return spill_bytes + (size_t)(key_cap + kTsGenCap) * 2 + (size_t)E * 4;
}
bool ts_fits(int64_t Lmax, int64_t E) { return ts_smem_bytes(Lmax, E) <= 196 * 1024; }
int tp_key_cap(int64_t Lmax) { return (int)(((Lmax + 7) & ~7ll) + 136); }  // read slack of the streamed selection
size_t tp_smem_bytes(int64_t Lmax, int64_t E, int64_t C) {  // topq_pipe_kernel: score row, 2 keys, 2 winners, 3 metas
  return (size_t)((Lmax + 7) & ~7ll) * 2 + (size_t)tp_key_cap(Lmax) * 2 * 2 + (size_t)E * 4 * 2 + (size_t)(6 * C + 1) * 4 * 3;
}
// 214 KB of dynamic shared memory with the kernel's 12.4 KB of static arrays stays under the 227 KB a
// CTA can have (rows up to about 35.3K positions at C = 64, E = 216)
bool tp_fits(int64_t Lmax, int64_t E, int64_t C) { return tp_smem_bytes(Lmax, E, C) <= 214 * 1024; }
int64_t ck_stride(int64_t Lmax) { return (Lmax + 7) & ~7ll; }
}  // namespace
}  // namespace oa

extern "C" int oa_topq_variant(int64_t Lmax, int64_t E, int64_t C) {
  if (oa::tp_fits(Lmax, E, C)) return 0;
  return oa::ts_fits(Lmax, E) ? 1 : 2;
}

extern "C" size_t oa_topq_workspace_bytes(int64_t R, int64_t Lmax, int64_t E) {
  if (R <= 0 || Lmax <= 0 || oa::ts_fits(Lmax, E)) return 0;
  return (size_t)(R * oa::ck_stride(Lmax) + 1024) * sizeof(uint16_t);
}

extern "C" int oa_topq(const void* scores, int64_t score_stride, int64_t R, int64_t Lmax, int64_t C,
                       const int32_t* mem, const int32_t* cstart, const int32_t* clen, const int32_t* asg,
                       const int32_t* reclist, const int32_t* reccnt, int rmax, const float* quota, int64_t E,
                       const int32_t* n_dev, const int32_t* n0_dev, int32_t* exp_idx, int32_t* status,
                       void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "oa_topq";
  OA_REQUIRE(R > 0 && Lmax > 0 && Lmax < (1 << 30) && C > 0 && C <= kMaxC && E > 0 && E < (1 << 23),
             "%s: bad sizes", fn);
  OA_REQUIRE(score_stride >= ((Lmax + 7) & ~7ll) && score_stride % 8 == 0 && oa_aligned16(scores),
             "%s: score rows must be 16-byte aligned and hold Lmax rounded up to 8", fn);
  OA_REQUIRE(scores && mem && cstart && clen && asg && quota && n_dev && n0_dev && exp_idx, "%s: null pointer", fn);
  OA_REQUIRE(reclist == nullptr || (reccnt != nullptr && rmax > 0), "%s: reclist needs reccnt and rmax", fn);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t spill_bytes = (size_t)((Lmax + 7) & ~7ll) * 2;
  if (tp_fits(Lmax, E, C)) {  // pipelined persistent kernel: the score row and two key buffers fit
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    TopqArgs a{static_cast<const uint16_t*>(scores), score_stride, (int)Lmax, (int)C, (int)E, rmax, 1, mem, cstart,
               clen, asg, reclist, reccnt, quota, n_dev, n0_dev, exp_idx, status};
    const size_t smem_tp = tp_smem_bytes(Lmax, E, C);
    if (int rc0 = oa_smem_opt_in(reinterpret_cast<const void*>(topq_pipe_kernel), smem_tp, fn)) return rc0;
    // fewer rows than SMs: split each row's clusters over up to 4 CTAs
    const int parts = (int)std::max<int64_t>(1, std::min<int64_t>({4, sms / R, C}));
    const int grid = (int)std::min<int64_t>(R * parts, sms);
    topq_pipe_kernel<<<grid, kTpThreads, smem_tp, st>>>(a, (int)R, (int)spill_bytes, tp_key_cap(Lmax), parts);
    return oa_check_launch(fn);
  }
  if (ts_fits(Lmax, E)) {  // persistent streamed-key kernel: score row, member keys and generated keys fit
    const int key_cap = (int)(((Lmax + 7) & ~7ll) + 1040);  // list slack of the register path
    const size_t smem_ts = ts_smem_bytes(Lmax, E);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    TopqArgs a{static_cast<const uint16_t*>(scores), score_stride, (int)Lmax, (int)C, (int)E, rmax, 1, mem, cstart,
               clen, asg, reclist, reccnt, quota, n_dev, n0_dev, exp_idx, status};
    if (int rc0 = oa_smem_opt_in(reinterpret_cast<const void*>(topq_stream_kernel), smem_ts, fn)) return rc0;
    // fewer rows than SMs: split each row's clusters over up to 4 CTAs
    const int parts = (int)std::max<int64_t>(1, std::min<int64_t>({4, sms / R, C}));
    const int grid = (int)std::min<int64_t>(R * parts, sms);
    topq_stream_kernel<<<grid, kTsThreads, smem_ts, st>>>(a, (int)R, (int)spill_bytes, key_cap, parts);
    return oa_check_launch(fn);
  }
  TopqArgs a{static_cast<const uint16_t*>(scores), score_stride, (int)Lmax, (int)C, (int)E, rmax, 0, mem, cstart,
             clen, asg, reclist, reccnt, quota, n_dev, n0_dev, exp_idx, status};
  if (workspace != nullptr && workspace_bytes >= oa_topq_workspace_bytes(R, Lmax, E)) {
    // long rows: keys permuted into CSR order in the workspace, then selected from contiguous keys
    OA_REQUIRE(oa_aligned16(workspace), "%s: workspace must be 16-byte aligned", fn);
    uint16_t* ck = static_cast<uint16_t*>(workspace);
    const int64_t ckw = ck_stride(Lmax);
    const size_t smem = (size_t)kPmChunk * 2;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // fewer rows than SMs: each row's clusters are split over up to 4 CTAs in both kernels
    const int parts = (int)std::max<int64_t>(1, std::min<int64_t>({4, sms / R, C}));
    if (int rc0 = oa_smem_opt_in(reinterpret_cast<const void*>(topq_permute_kernel), smem, fn)) return rc0;
    topq_permute_kernel<<<(unsigned)(R * parts), kPmThreads, smem, st>>>(a, ck, ckw, parts);
    int rc = oa_check_launch(fn);
    if (rc != OA_OK) return rc;
    const size_t smem_ck = (size_t)kCkWarps * kCkWinSlots * sizeof(uint16_t);
    if (int rc2 = oa_smem_opt_in(reinterpret_cast<const void*>(topq_ck_kernel), smem_ck, fn)) return rc2;
    topq_ck_kernel<<<(unsigned)(R * parts), kCkThreads, smem_ck, st>>>(a, ck, ckw, parts);
    return oa_check_launch(fn);
  }
  const bool in_smem = spill_bytes <= 160 * 1024;  // larger rows read their keys from global memory
  a.smem_keys = in_smem ? 1 : 0;
  const size_t smem = in_smem ? spill_bytes : 16;
  if (int rc0 = oa_smem_opt_in(reinterpret_cast<const void*>(topq_kernel), smem, fn)) return rc0;
  topq_kernel<<<(unsigned)R, kTqThreads, smem, st>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_residual(const void* K, const void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C,
                           const int32_t* asg,
                           const int32_t* sel, int64_t n_sel, const int32_t* exp_idx, int64_t E, const float* Sk,
                           const float* Sv, const float* nt, const float* quota, void* kbar, void* vbar, float* logn,
                           int32_t* status, void* stream) {
  const char* fn = "oa_residual";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= kMaxC && E > 0, "%s: bad sizes", fn);
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(n_sel > 0 && n_sel + E <= kMaxRead, "%s: need 0 < n_sel and n_sel + E <= %d", fn, kMaxRead);
  OA_REQUIRE(K && V && asg && sel && exp_idx && Sk && Sv && nt && quota && kbar && vbar && logn, "%s: null pointer",
             fn);
  OA_REQUIRE(oa_aligned16(K) && oa_aligned16(V), "%s: K / V must be 16-byte aligned", fn);
  ResidArgs a{nullptr, 0, static_cast<const __nv_bfloat16*>(K), static_cast<const __nv_bfloat16*>(V), (int)Lmax,
              (int)C, (int)n_sel, (int)E, asg, sel, exp_idx, Sk, Sv, nt, quota, nullptr, static_cast<__nv_bfloat16*>(kbar),
              static_cast<__nv_bfloat16*>(vbar), logn, nullptr, 0, 0, 0.f, status};
  residual_kernel<false><<<(unsigned)(B * kG * hkv), kRW * 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_residual_flash(const void* q, int64_t q_stride, const void* K, const void* V, int64_t B, int64_t hkv,
                                 int64_t Lmax, int64_t C, const int32_t* asg, const int32_t* sel, int64_t n_sel,
                                 const int32_t* exp_idx, int64_t E, const float* Sk, const float* Sv, const float* nt,
                                 const float* quota, const float* zdot, void* kbar, void* vbar, float* logn, void* out,
                                 int64_t out_stride, int out_dtype, float sm_scale, int32_t* status, void* stream) {
  const char* fn = "oa_residual_flash";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= kMaxC && E > 0, "%s: bad sizes", fn);
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(n_sel > 0 && n_sel + E <= kMaxRead, "%s: need 0 < n_sel and n_sel + E <= %d", fn, kMaxRead);
  OA_REQUIRE(q && K && V && asg && sel && exp_idx && Sk && Sv && nt && quota && out, "%s: null pointer", fn);
  OA_REQUIRE((kbar == nullptr) == (vbar == nullptr), "%s: kbar and vbar are given together", fn);
  OA_REQUIRE(out_dtype == OA_BF16 || out_dtype == OA_F32, "%s: out_dtype must be OA_BF16 or OA_F32", fn);
  OA_REQUIRE(oa_aligned16(K) && oa_aligned16(V), "%s: K / V must be 16-byte aligned", fn);
  ResidArgs a{static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<const __nv_bfloat16*>(K),
              static_cast<const __nv_bfloat16*>(V), (int)Lmax, (int)C, (int)n_sel, (int)E, asg, sel, exp_idx, Sk, Sv,
              nt, quota, zdot, static_cast<__nv_bfloat16*>(kbar), static_cast<__nv_bfloat16*>(vbar), logn, out,
              out_stride, out_dtype == OA_F32 ? 1 : 0, sm_scale * kLog2e, status};
  if (kbar == nullptr && logn == nullptr) {
    OA_REQUIRE(oa_aligned16(q) && q_stride % 8 == 0, "%s: q rows must be 16-byte aligned", fn);
    OA_REQUIRE(oa_aligned16(Sk) && oa_aligned16(Sv), "%s: Sk / Sv must be 16-byte aligned", fn);
    const size_t smem = proxy_flash_smem((int)(n_sel + E), (int)C);
    const int64_t R = B * kG * hkv;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (R * 2 <= sms) {  // few rows: each row on a cluster of 4 CTAs (distributed shared memory)
      constexpr int kN = 4;
      if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(proxy_flash_kernel<kN>), smem, fn)) return rc;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(R * kN));
      cfg.blockDim = dim3(kPF);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = static_cast<cudaStream_t>(stream);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = kN;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const cudaError_t e = cudaLaunchKernelEx(&cfg, proxy_flash_kernel<kN>, a);
      if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: cluster launch failed: %s", fn, cudaGetErrorString(e));
    } else {
      if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(proxy_flash_kernel<1>), smem, fn)) return rc;
      proxy_flash_kernel<1><<<(unsigned)R, kPF, smem, static_cast<cudaStream_t>(stream)>>>(a);
    }
  } else {
    residual_kernel<true><<<(unsigned)(B * kG * hkv), kRW * 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  }
  return oa_check_launch(fn);
}
