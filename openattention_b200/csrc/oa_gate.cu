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
#include "../../include/openattention_b200.h"

namespace oa {
namespace {

constexpr int kMaxC = 256;
constexpr int kGateThreads = 256;

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
};

__global__ void __launch_bounds__(kGateThreads) errorgate_waterfill_kernel(const GateArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kv = r / kG;
  const int C = a.C;
  __shared__ float s_score[kMaxC], s_nt[kMaxC], s_w[kMaxC], s_cap[kMaxC], s_ratio[kMaxC], s_qb[kMaxC];
  __shared__ float s_cex[kMaxC], s_wsuf[kMaxC];
  __shared__ int s_ord[kMaxC], s_rank2[kMaxC];
  __shared__ int s_selc[512];
  __shared__ int s_selt[512];
  __shared__ float s_red[8];
  __shared__ int s_redi[8];
  for (int j = tid; j < a.NS; j += blockDim.x) {
    const int t = a.sel[(int64_t)r * a.NS + j];
    s_selt[j] = t;
    s_selc[j] = (t >= 0 && t < a.Lmax) ? a.asg[(int64_t)r * a.Lmax + t] : -1;
  }
  float qv[4], q2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qv[i] = __bfloat162float(a.q[(int64_t)r * a.q_stride + lane + 32 * i]);
    q2[i] = __fmul_rn(qv[i], qv[i]);
  }
  __syncthreads();
  // ---- ErrorGate: warp per cluster
  for (int c = warp; c < C; c += kGateThreads / 32) {
    float skt[4], sk2t[4];
    const int64_t base = ((int64_t)r * C + c) * kD;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      skt[i] = a.Sk[base + lane + 32 * i];
      sk2t[i] = a.Sk2[base + lane + 32 * i];
    }
    float ntc = a.nb[(int64_t)r * C + c];
    for (int j = 0; j < a.NS; ++j) {
      if (s_selc[j] != c) continue;
      const __nv_bfloat16* kr = a.K + ((int64_t)kv * a.Lmax + s_selt[j]) * kD;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float kf = __bfloat162float(kr[lane + 32 * i]);
        skt[i] = __fsub_rn(skt[i], kf);
        sk2t[i] = __fsub_rn(sk2t[i], __fmul_rn(kf, kf));
      }
      ntc = __fsub_rn(ntc, 1.f);
    }
    const float inv = __fdiv_rn(1.f, fmaxf(ntc, 1.f));
    float kb[4], var[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      kb[i] = __fmul_rn(skt[i], inv);
      const float p1 = __fmul_rn(sk2t[i], inv);
      const float p2 = __fmul_rn(kb[i], kb[i]);
      var[i] = fmaxf(__fsub_rn(p1, p2), 0.f);
    }
    const float zd = warp_tree_dot(qv, kb);
    const float sd = warp_tree_dot(q2, var);
    if (lane == 0) {
      const float zbar = __fmul_rn(0.08838834764831845f, zd);
      const float s2 = __fmul_rn(0.0078125f, sd);
      const float lg = ln_f(fmaxf(ntc, 1.f));
      const float er = erf_f(__fmul_rn(__fsqrt_rn(s2), 0.70710677f));
      const float le = ln_f(fmaxf(er, 1e-30f));
      float sc = __fadd_rn(zbar, lg);
      sc = __fadd_rn(sc, __fmul_rn(0.5f, s2));
      sc = __fadd_rn(sc, le);
      s_score[c] = sc;
      s_nt[c] = ntc;
    }
  }
  __syncthreads();
  // ---- water-filling (thread c <-> cluster c)
  const int c = tid;
  const bool act = c < C;
  const bool live = act && s_nt[c] > 1.f;
  const float sm = live ? s_score[c] : -INFINITY;
  float smax = sm;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, off));
  if (lane == 0) s_red[warp] = smax;
  __syncthreads();
  smax = s_red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) smax = fmaxf(smax, s_red[w]);
  float w = 0.f, cap = 0.f, ratio = INFINITY;
  if (act) {
    w = live ? exp_f(__fsub_rn(sm, smax)) : 0.f;
    cap = live ? s_nt[c] : 0.f;
    ratio = w > 0.f ? __fdiv_rn(cap, fmaxf(w, 1e-30f)) : INFINITY;
    s_w[c] = w;
    s_cap[c] = cap;
    s_ratio[c] = ratio;
  }
  __syncthreads();
  float tot = 0.f;  // integer-valued: exact in any order
  for (int j = 0; j < C; ++j) tot = __fadd_rn(tot, s_cap[j]);
  if (act) {
    // rank by (ratio asc, cluster asc); rank by (score desc, cluster asc)
    int r1 = 0, r2 = 0;
    for (int j = 0; j < C; ++j) {
      const float rj = s_ratio[j];
      r1 += (rj < ratio || (rj == ratio && j < c)) ? 1 : 0;
      const bool lj = s_nt[j] > 1.f;
      const float sj = lj ? s_score[j] : -INFINITY;
      r2 += (sj > sm || (sj == sm && j < c)) ? 1 : 0;
    }
    s_ord[r1] = c;
    s_rank2[c] = r2;
  }
  __syncthreads();
  if (act) {  // exclusive prefix of the caps in ratio order (integers)
    float cex = 0.f;
    for (int j = 0; j < c; ++j) cex = __fadd_rn(cex, s_cap[s_ord[j]]);
    s_cex[c] = cex;  // indexed by sorted position c
  }
  if (tid == 0) {  // suffix sums of the weights in ratio order, accumulated in double from the end
    double acc = 0.0;
    for (int j = C - 1; j >= 0; --j) {
      acc = __dadd_rn(acc, (double)s_w[s_ord[j]]);
      s_wsuf[j] = __double2float_rn(acc);
    }
  }
  __syncthreads();
  int jj = 0x7fffffff;
  if (act) {
    const float ws = s_wsuf[c];
    const float f = ws > 0.f ? __fadd_rn(s_cex[c], __fmul_rn(s_ratio[s_ord[c]], ws)) : INFINITY;
    if (f >= a.E) jj = c;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) jj = min(jj, __shfl_xor_sync(0xffffffffu, jj, off));
  if (lane == 0) s_redi[warp] = jj;
  __syncthreads();
  jj = s_redi[0];
#pragma unroll
  for (int v = 1; v < 8; ++v) jj = min(jj, s_redi[v]);
  if (jj == 0x7fffffff) jj = 0;
  const float lam = __fdiv_rn(__fsub_rn(a.E, s_cex[jj]), fmaxf(s_wsuf[jj], 1e-30f));
  float qb = 0.f;
  if (act) {
    qb = fminf(cap, floorf(__fmul_rn(lam, w)));
    if (tot <= a.E) qb = cap;
    s_qb[c] = qb;
  }
  __syncthreads();
  float sumq = 0.f;
  for (int j = 0; j < C; ++j) sumq = __fadd_rn(sumq, s_qb[j]);
  const float rem = fmaxf(__fsub_rn(fminf(tot, a.E), sumq), 0.f);
  if (act) {
    const bool room = qb < cap;
    int before = 0;  // clusters with room ranked ahead by (score desc, cluster asc)
    const int my = s_rank2[c];
    for (int j = 0; j < C; ++j) before += (s_qb[j] < s_cap[j] && s_rank2[j] < my) ? 1 : 0;
    const float add = (room && (float)before < rem) ? 1.f : 0.f;
    a.quota[(int64_t)r * C + c] = __fadd_rn(qb, add);
    a.nt[(int64_t)r * C + c] = s_nt[c];
    a.score[(int64_t)r * C + c] = s_score[c];
  }
}

// ------------------------------------------------------------------------ within-cluster top-q
constexpr int kTopqWarps = 8;
constexpr int kCap = 1536;  // candidates held in shared memory per warp (larger clusters stream)

struct TopqArgs {
  const uint16_t* scores;
  int64_t sw;
  int Lmax, C, E, rmax;
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
};

__device__ __forceinline__ uint32_t ukey16(uint32_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }

// Candidate i of cluster c (members in CSR order, then generated tokens in position order).
struct CandSrc {
  const int32_t* mem;   // member list of (r, c)
  int nmem;
  const int32_t* rec;   // generated-token list, or nullptr to scan [n0, n)
  int nrec;
  const int32_t* asg_r;
  int n0, n, c;
};

__global__ void __launch_bounds__(kTopqWarps * 32) topq_kernel(const TopqArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = a.C;
  const int n = __ldg(a.n_dev), n0 = __ldg(a.n0_dev);
  __shared__ int s_base[kMaxC + 1];
  __shared__ int s_next;
  extern __shared__ __align__(16) unsigned char topq_smem[];
  int32_t* s_tok = reinterpret_cast<int32_t*>(topq_smem);                              // [warps][kCap]
  int* s_hist = reinterpret_cast<int*>(s_tok + kTopqWarps * kCap);                      // [warps][256]
  uint16_t* s_key = reinterpret_cast<uint16_t*>(s_hist + kTopqWarps * 256);              // [warps][kCap]
  if (tid == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      s_base[c] = run;
      run += (int)a.quota[(int64_t)r * C + c];
    }
    s_base[C] = run;
    s_next = 0;
  }
  __syncthreads();
  int32_t* out = a.exp + (int64_t)r * a.E;
  for (int i = s_base[C] + tid; i < a.E; i += blockDim.x) out[i] = -1;
  const uint16_t* sr = a.scores + (int64_t)r * a.sw;
  const int32_t* asg_r = a.asg + (int64_t)r * a.Lmax;
  uint16_t* keys = s_key + warp * kCap;
  int32_t* toks = s_tok + warp * kCap;
  int* hist = s_hist + warp * 256;
  while (true) {
    int c = 0;
    if (lane == 0) c = atomicAdd(&s_next, 1);
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= C) break;
    const int q = s_base[c + 1] - s_base[c];
    if (q <= 0) continue;
    const int base = s_base[c];
    const int64_t rc = (int64_t)r * C + c;
    const int nmem = a.clen[rc];
    const int32_t* mem = a.mem + (int64_t)r * a.Lmax + a.cstart[rc];
    const int cnt = a.reclist ? a.reccnt[rc] : 0x7fffffff;
    const bool use_list = a.reclist != nullptr && cnt <= a.rmax;
    const int32_t* rec = use_list ? a.reclist + rc * a.rmax : nullptr;
    const int ngen_scan = max(0, n - n0);
    // enumerate candidates in order: members, then generated tokens (list, or scan of [n0, n))
    // chunks of 32; f(tok, key) is applied to each candidate in order
    auto for_each = [&](auto&& f) {
      for (int i0 = 0; i0 < nmem; i0 += 32) {
        const int i = i0 + lane;
        const bool v = i < nmem;
        const int t = v ? mem[i] : 0;
        const uint32_t k = v ? ukey16(sr[t]) : 0u;
        f(v, t, k);
      }
      if (use_list) {
        for (int i0 = 0; i0 < cnt; i0 += 32) {
          const int i = i0 + lane;
          const bool v = i < cnt;
          const int t = v ? rec[i] : 0;
          const uint32_t k = v ? ukey16(sr[t]) : 0u;
          f(v, t, k);
        }
      } else {
        for (int i0 = 0; i0 < ngen_scan; i0 += 32) {
          const int t = n0 + i0 + lane;
          const bool v = (i0 + lane < ngen_scan) && asg_r[t] == c;
          const uint32_t k = v ? ukey16(sr[t]) : 0u;
          f(v, t, k);
        }
      }
    };
    const int total = nmem + (use_list ? cnt : ngen_scan);
    const bool in_smem = total <= kCap;
    int m = 0;  // compacted candidate count (in smem mode)
    if (in_smem) {
      for_each([&](bool v, int t, uint32_t k) {
        const unsigned bal = __ballot_sync(0xffffffffu, v);
        const int pos = m + __popc(bal & ((1u << lane) - 1u));
        if (v) {
          keys[pos] = (uint16_t)k;
          toks[pos] = t;
        }
        m += __popc(bal);
      });
      __syncwarp();
    }
    // two 8-bit radix passes: threshold key T = the q-th largest key
    int above = 0, hi = 0, lo = 0;
    for (int pass = 0; pass < 2; ++pass) {
      for (int b = lane; b < 256; b += 32) hist[b] = 0;
      __syncwarp();
      auto add = [&](bool v, int t, uint32_t k) {
        if (v && (pass == 0 || (int)(k >> 8) == hi)) atomicAdd(&hist[pass == 0 ? (k >> 8) : (k & 255)], 1);
      };
      if (in_smem) {
        for (int i = lane; i < m; i += 32) add(true, 0, keys[i]);
      } else {
        for_each(add);
      }
      __syncwarp();
      // find the bin (from the top) where the running count reaches q: lane l owns bins 255-8l..248-8l
      int cnt8[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt8[i] = hist[255 - 8 * lane - i];
        s += cnt8[i];
      }
      int incl = s;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const int excl = incl - s;
      const int need = q - above;
      int found_bin = -1, found_above = 0;
      if (excl < need && incl >= need) {
        int run = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (found_bin < 0 && run + cnt8[i] >= need) {
            found_bin = 255 - 8 * lane - i;
            found_above = run;
          }
          run += cnt8[i];
        }
      }
      const unsigned who = __ballot_sync(0xffffffffu, found_bin >= 0);
      const int src = who ? (__ffs(who) - 1) : 0;
      const int fb = __shfl_sync(0xffffffffu, found_bin, src);
      const int fa = __shfl_sync(0xffffffffu, found_above, src);
      if (pass == 0) hi = fb < 0 ? 0 : fb;
      else lo = fb < 0 ? 0 : fb;
      above += fa;
      __syncwarp();
    }
    const uint32_t T = ((uint32_t)hi << 8) | (uint32_t)lo;
    const int need_eq = q - above;
    // collect in candidate order: keys > T, and the first need_eq keys == T
    int taken = 0, ties = 0;
    auto collect = [&](bool v, int t, uint32_t k) {
      const bool gt = v && k > T;
      const bool eq = v && k == T;
      const unsigned beq = __ballot_sync(0xffffffffu, eq);
      const int er = ties + __popc(beq & ((1u << lane) - 1u));
      const bool take = gt || (eq && er < need_eq);
      const unsigned bt = __ballot_sync(0xffffffffu, take);
      const int slot = taken + __popc(bt & ((1u << lane) - 1u));
      if (take && slot < q && base + slot < a.E) out[base + slot] = t;
      taken += __popc(bt);
      ties += __popc(beq);
    };
    if (in_smem) {
      for (int i0 = 0; i0 < m; i0 += 32) {
        const int i = i0 + lane;
        const bool v = i < m;
        collect(v, v ? toks[i] : 0, v ? keys[i] : 0u);
      }
    } else {
      for_each(collect);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------ residual proxies
struct ResidArgs {
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
  __nv_bfloat16* kbar;
  __nv_bfloat16* vbar;
  float* logn;
};

__global__ void __launch_bounds__(kGateThreads) residual_kernel(const ResidArgs a) {
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kv = r / kG;
  const int C = a.C;
  __shared__ int s_base[kMaxC + 1];
  __shared__ int s_selc[512], s_selt[512];
  for (int j = tid; j < a.NS; j += blockDim.x) {
    const int t = a.sel[(int64_t)r * a.NS + j];
    s_selt[j] = t;
    s_selc[j] = (t >= 0 && t < a.Lmax) ? a.asg[(int64_t)r * a.Lmax + t] : -1;
  }
  if (tid == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      s_base[c] = run;
      run += (int)a.quota[(int64_t)r * C + c];
    }
    s_base[C] = run;
  }
  __syncthreads();
  const __nv_bfloat16* Kr = a.K + (int64_t)kv * a.Lmax * kD;
  const __nv_bfloat16* Vr = a.V + (int64_t)kv * a.Lmax * kD;
  for (int c = warp; c < C; c += kGateThreads / 32) {
    const int64_t base = ((int64_t)r * C + c) * kD;
    float sk[4], sv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sk[i] = a.Sk[base + lane + 32 * i];
      sv[i] = a.Sv[base + lane + 32 * i];
    }
    auto sub = [&](int t) {
      const __nv_bfloat16* kr = Kr + (int64_t)t * kD;
      const __nv_bfloat16* vr = Vr + (int64_t)t * kD;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sk[i] = __fsub_rn(sk[i], __bfloat162float(kr[lane + 32 * i]));
        sv[i] = __fsub_rn(sv[i], __bfloat162float(vr[lane + 32 * i]));
      }
    };
    for (int j = 0; j < a.NS; ++j)
      if (s_selc[j] == c) sub(s_selt[j]);
    const int e0 = s_base[c], e1 = min(s_base[c + 1], a.E);
    for (int s = e0; s < e1; ++s) {
      const int t = a.exp[(int64_t)r * a.E + s];
      if (t >= 0 && t < a.Lmax) sub(t);
    }
    const float nr = __fsub_rn(a.nt[(int64_t)r * C + c], a.quota[(int64_t)r * C + c]);
    const float inv = __fdiv_rn(1.f, fmaxf(nr, 1.f));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a.kbar[base + lane + 32 * i] = __float2bfloat16_rn(__fmul_rn(sk[i], inv));
      a.vbar[base + lane + 32 * i] = __float2bfloat16_rn(__fmul_rn(sv[i], inv));
    }
    if (lane == 0) a.logn[(int64_t)r * C + c] = nr > 0.5f ? ln_f(fmaxf(nr, 1.f)) : -INFINITY;
  }
}

}  // namespace
}  // namespace oa

using namespace oa;

extern "C" int oa_errorgate_waterfill(const void* q, int64_t q_stride, const void* K, int64_t B, int64_t Lmax,
                                      int64_t C, const int32_t* asg, const int32_t* sel, int64_t n_sel,
                                      const float* Sk, const float* Sk2, const float* nb, float E, float* score,
                                      float* nt, float* quota, void* stream) {
  const char* fn = "oa_errorgate_waterfill";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= kMaxC, "%s: need 0 < C <= %d (C=%lld)", fn, kMaxC, (long long)C);
  OA_REQUIRE(n_sel > 0 && n_sel <= 512, "%s: n_sel=%lld outside [1, 512]", fn, (long long)n_sel);
  OA_REQUIRE(q && K && asg && sel && Sk && Sk2 && nb && score && nt && quota, "%s: null pointer", fn);
  OA_REQUIRE(E >= 0.f, "%s: negative budget", fn);
  GateArgs a{static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<const __nv_bfloat16*>(K), (int)Lmax, (int)C,
             (int)n_sel, asg, sel, Sk, Sk2, nb, E, score, nt, quota};
  errorgate_waterfill_kernel<<<(unsigned)(B * kHQ), kGateThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_topq(const void* scores, int64_t score_stride, int64_t R, int64_t Lmax, int64_t C,
                       const int32_t* mem, const int32_t* cstart, const int32_t* clen, const int32_t* asg,
                       const int32_t* reclist, const int32_t* reccnt, int rmax, const float* quota, int64_t E,
                       const int32_t* n_dev, const int32_t* n0_dev, int32_t* exp_idx, void* stream) {
  const char* fn = "oa_topq";
  OA_REQUIRE(R > 0 && Lmax > 0 && C > 0 && C <= kMaxC && E > 0, "%s: bad sizes", fn);
  OA_REQUIRE(score_stride >= Lmax, "%s: score stride < Lmax", fn);
  OA_REQUIRE(scores && mem && cstart && clen && asg && quota && n_dev && n0_dev && exp_idx, "%s: null pointer", fn);
  OA_REQUIRE(reclist == nullptr || (reccnt != nullptr && rmax > 0), "%s: reclist needs reccnt and rmax", fn);
  TopqArgs a{static_cast<const uint16_t*>(scores), score_stride, (int)Lmax, (int)C, (int)E, rmax, mem, cstart, clen,
             asg, reclist, reccnt, quota, n_dev, n0_dev, exp_idx};
  constexpr size_t smem = (size_t)kTopqWarps * (kCap * 6 + 256 * 4);
  static bool attr_set = false;  // idempotent attribute, set once per process
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(topq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
    attr_set = true;
  }
  topq_kernel<<<(unsigned)R, kTopqWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}

extern "C" int oa_residual(const void* K, const void* V, int64_t B, int64_t Lmax, int64_t C, const int32_t* asg,
                           const int32_t* sel, int64_t n_sel, const int32_t* exp_idx, int64_t E, const float* Sk,
                           const float* Sv, const float* nt, const float* quota, void* kbar, void* vbar, float* logn,
                           void* stream) {
  const char* fn = "oa_residual";
  OA_REQUIRE(B > 0 && Lmax > 0 && C > 0 && C <= kMaxC && E > 0, "%s: bad sizes", fn);
  OA_REQUIRE(n_sel > 0 && n_sel <= 512, "%s: n_sel outside [1, 512]", fn);
  OA_REQUIRE(K && V && asg && sel && exp_idx && Sk && Sv && nt && quota && kbar && vbar && logn, "%s: null pointer",
             fn);
  ResidArgs a{static_cast<const __nv_bfloat16*>(K), static_cast<const __nv_bfloat16*>(V), (int)Lmax, (int)C,
              (int)n_sel, (int)E, asg, sel, exp_idx, Sk, Sv, nt, quota, static_cast<__nv_bfloat16*>(kbar),
              static_cast<__nv_bfloat16*>(vbar), logn};
  residual_kernel<<<(unsigned)(B * kHQ), kGateThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return oa_check_launch(fn);
}
