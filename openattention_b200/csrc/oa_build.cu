// Per-request index build (prefill side) on sm_100a: QGS codes, QGC projection + column means,
// Lloyd iterations (assignment, stable CSR, centroid update) and the per-cluster sums.
//
// Restates methods_eager.Ours.build (inference/methods_eager.py:519-555) and the fast build of
// inference/ours_fastbuild.py:253-304 (_k_km_assign, _k_km_update, _k_cluster_sums) with
// deterministic reductions: sums run sequentially over members in position order (the order of the
// eager reference's CPU scatter_add), column means accumulate in double per 256-token tile, then
// sequentially over tiles.  No floating-point atomics.
//
// All entry points work on ONE request: K, V are (8, Lmax, 128) bf16; the 32 query heads of the
// request index the state arrays' leading dimension.
#include "oa_common.cuh"
#include "../../include/openattention_b200.h"

namespace oa {
namespace {

constexpr int kBT = 256;  // tokens per block / per column-mean tile

__device__ __forceinline__ void load_row(const __nv_bfloat16* p, uint32_t (&w)[64]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint4 v = __ldg(q + i);
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}
__device__ __forceinline__ float row_at(const uint32_t (&w)[64], int d) {
  return (d & 1) ? bf_hi(w[d >> 1]) : bf_lo(w[d >> 1]);
}

// ---------------------------------------------------------------- QGS codes
// z[h, t, j] = sum_d k.U (d ascending, fma); pass 1 takes amax_t |z| per (h, j), pass 2 quantises.
template <bool QUANT>
__global__ void __launch_bounds__(kBT) build_codes_kernel(const __nv_bfloat16* K, int Lmax, int T, const float* U,
                                                          uint32_t* amax, const float* scale, int8_t* codes) {
  const int h = blockIdx.y;
  const int t = blockIdx.x * kBT + threadIdx.x;
  __shared__ float sU[kD * kRQ];
  for (int i = threadIdx.x; i < kD * kRQ; i += kBT) sU[i] = U[(int64_t)h * kD * kRQ + i];
  __syncthreads();
  if (t >= T) return;
  uint32_t w[64];
  load_row(K + ((int64_t)h * Lmax + t) * kD, w);
  float acc[kRQ];
#pragma unroll
  for (int j = 0; j < kRQ; ++j) acc[j] = 0.f;
#pragma unroll
  for (int d = 0; d < kD; ++d) {
    const float kd = row_at(w, d);
#pragma unroll
    for (int j = 0; j < kRQ; ++j) acc[j] = __fmaf_rn(kd, sU[d * kRQ + j], acc[j]);
  }
  if (!QUANT) {
#pragma unroll
    for (int j = 0; j < kRQ; ++j) atomicMax(&amax[h * kRQ + j], __float_as_uint(fabsf(acc[j])));
  } else {
    int8_t out[kRQ];
#pragma unroll
    for (int j = 0; j < kRQ; ++j) {
      float c = rintf(__fdiv_rn(acc[j], scale[h * kRQ + j]));
      out[j] = (int8_t)fminf(fmaxf(c, -127.f), 127.f);
    }
    uint4* dst = reinterpret_cast<uint4*>(codes + ((int64_t)h * Lmax + t) * kRQ);
    dst[0] = *reinterpret_cast<uint4*>(&out[0]);
    dst[1] = *reinterpret_cast<uint4*>(&out[16]);
  }
}

__global__ void build_scale_kernel(const uint32_t* amax, float* scale, int n) {
  const int i = threadIdx.x + blockIdx.x * blockDim.x;
  if (i < n) scale[i] = fmaxf(__fdiv_rn(__uint_as_float(amax[i]), 127.f), 1e-12f);
}

// ---------------------------------------------------------------- QGC projection
// zp[h, t, c] = bf16(sum_d k.W[h] (d ascending, fma)); per-tile double partial sums (sequential in t)
__global__ void __launch_bounds__(kBT) project_kernel(const __nv_bfloat16* K, int Lmax, int T, const __nv_bfloat16* W,
                                                      float* zP, double* part) {
  const int h = blockIdx.y;
  const int tile = blockIdx.x;
  const int t = tile * kBT + threadIdx.x;
  __shared__ float sW[kD * kRC];
  __shared__ float sZ[kBT][kRC + 1];
  for (int i = threadIdx.x; i < kD * kRC; i += kBT) sW[i] = __bfloat162float(W[(int64_t)h * kD * kRC + i]);
  __syncthreads();
  if (t < T) {
    uint32_t w[64];
    load_row(K + ((int64_t)(h / kG) * Lmax + t) * kD, w);
    float acc[kRC];
#pragma unroll
    for (int c = 0; c < kRC; ++c) acc[c] = 0.f;
#pragma unroll
    for (int d = 0; d < kD; ++d) {
      const float kd = row_at(w, d);
#pragma unroll
      for (int c = 0; c < kRC; ++c) acc[c] = __fmaf_rn(kd, sW[d * kRC + c], acc[c]);
    }
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      const float zb = bf_round(acc[c]);
      sZ[threadIdx.x][c] = zb;
      zP[((int64_t)h * T + t) * kRC + c] = zb;
    }
  }
  __syncthreads();
  if (threadIdx.x < kRC) {
    const int c = threadIdx.x;
    double s = 0.0;
    const int nt = min(kBT, T - tile * kBT);
    for (int i = 0; i < nt; ++i) s = __dadd_rn(s, (double)sZ[i][c]);
    part[((int64_t)h * gridDim.x + tile) * kRC + c] = s;
  }
}

__global__ void colmean_kernel(const double* part, int ntiles, int T, float* colmean, int nq) {
  const int i = threadIdx.x + blockIdx.x * blockDim.x;  // h * 16 + c
  if (i >= nq * kRC) return;
  const int h = i / kRC, c = i % kRC;
  double s = 0.0;
  for (int tl = 0; tl < ntiles; ++tl) s = __dadd_rn(s, part[((int64_t)h * ntiles + tl) * kRC + c]);
  colmean[i] = __double2float_rn(__ddiv_rn(s, (double)T));
}

__global__ void center_kernel(float* zP, int T, const float* colmean, int nq) {
  const int64_t i = threadIdx.x + (int64_t)blockIdx.x * blockDim.x;
  if (i >= (int64_t)nq * T * kRC) return;
  const int c = (int)(i % kRC);
  const int h = (int)(i / ((int64_t)T * kRC));
  zP[i] = __fsub_rn(zP[i], colmean[h * kRC + c]);
}

// ---------------------------------------------------------------- Lloyd assignment
// dist = bf16(bf16(zb . cb) - half), zb = bf16(zP), cb = bf16(cent), half = bf16(0.5 sum_c cent_c^2);
// argmax over clusters, ties -> lower id
__global__ void __launch_bounds__(kBT) kmeans_assign_kernel(const float* zP, int T, int C, const float* cent,
                                                            int32_t* asg, int64_t asg_stride) {
  extern __shared__ float sm[];
  float* cb = sm;             // C * 16
  float* half = sm + C * kRC;  // C
  const int h = blockIdx.y;
  for (int i = threadIdx.x; i < C; i += kBT) {
    float nrm = 0.f;
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      const float x = cent[((int64_t)h * C + i) * kRC + c];
      cb[i * kRC + c] = bf_round(x);
      nrm = __fadd_rn(nrm, __fmul_rn(x, x));
    }
    half[i] = bf_round(__fmul_rn(0.5f, nrm));
  }
  __syncthreads();
  const int t = blockIdx.x * kBT + threadIdx.x;
  if (t >= T) return;
  float zb[kRC];
  const float4* zp4 = reinterpret_cast<const float4*>(zP + ((int64_t)h * T + t) * kRC);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = zp4[i];
    zb[4 * i] = bf_round(v.x);
    zb[4 * i + 1] = bf_round(v.y);
    zb[4 * i + 2] = bf_round(v.z);
    zb[4 * i + 3] = bf_round(v.w);
  }
  int best = 0;
  float bestv = -INFINITY;
  for (int i = 0; i < C; ++i) {
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < kRC; ++c) acc = __fmaf_rn(zb[c], cb[i * kRC + c], acc);
    const float dd = bf_round(__fsub_rn(bf_round(acc), half[i]));
    if (dd > bestv) {
      bestv = dd;
      best = i;
    }
  }
  asg[(int64_t)h * asg_stride + t] = best;
}

// ---------------------------------------------------------------- stable CSR (counting sort)
__global__ void __launch_bounds__(kBT) csr_count_kernel(const int32_t* asg, int64_t asg_stride, int T, int C,
                                                        int32_t* tilecnt) {
  const int h = blockIdx.y, tile = blockIdx.x;
  extern __shared__ int hc[];
  for (int i = threadIdx.x; i < C; i += kBT) hc[i] = 0;
  __syncthreads();
  const int t = tile * kBT + threadIdx.x;
  if (t < T) atomicAdd(&hc[asg[(int64_t)h * asg_stride + t]], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < C; i += kBT) tilecnt[((int64_t)h * gridDim.x + tile) * C + i] = hc[i];
}

__global__ void csr_offsets_kernel(int32_t* tilecnt, int ntiles, int C, int32_t* cstart, int32_t* clen) {
  // one block per head; thread c turns its column of tile counts into tile offsets
  const int h = blockIdx.x;
  __shared__ int s_len[1024];
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    int run = 0;
    for (int tl = 0; tl < ntiles; ++tl) {
      int32_t* p = &tilecnt[((int64_t)h * ntiles + tl) * C + c];
      const int v = *p;
      *p = run;  // exclusive prefix within the cluster
      run += v;
    }
    s_len[c] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      cstart[h * C + c] = run;
      clen[h * C + c] = s_len[c];
      run += s_len[c];
    }
  }
}

__global__ void __launch_bounds__(kBT) csr_place_kernel(const int32_t* asg, int64_t asg_stride, int T, int C,
                                                        const int32_t* tileoff, const int32_t* cstart, int32_t* mem,
                                                        int64_t mem_stride) {
  const int h = blockIdx.y, tile = blockIdx.x;
  __shared__ int sa[kBT];
  const int t = tile * kBT + threadIdx.x;
  sa[threadIdx.x] = t < T ? asg[(int64_t)h * asg_stride + t] : -1;
  __syncthreads();
  if (t >= T) return;
  const int a = sa[threadIdx.x];
  int rank = 0;
  for (int i = 0; i < (int)threadIdx.x; ++i) rank += (sa[i] == a) ? 1 : 0;
  const int slot = cstart[h * C + a] + tileoff[((int64_t)h * gridDim.x + tile) * C + a] + rank;
  mem[(int64_t)h * mem_stride + slot] = t;
}

// ---------------------------------------------------------------- Lloyd update
// cent_i = (sum of member zP in position order) / count; empty -> zP[init_i]; nb = count
__global__ void kmeans_update_kernel(const float* zP, int T, int C, const int32_t* mem, int64_t mem_stride,
                                     const int32_t* cstart, const int32_t* clen, const int64_t* init, float* cent,
                                     float* nb) {
  const int h = blockIdx.y;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // i * 16 + c
  if (idx >= C * kRC) return;
  const int i = idx / kRC, c = idx % kRC;
  const int st = cstart[h * C + i], len = clen[h * C + i];
  const int32_t* mp = mem + (int64_t)h * mem_stride + st;
  float acc = 0.f;
  for (int j = 0; j < len; ++j) acc = __fadd_rn(acc, zP[((int64_t)h * T + mp[j]) * kRC + c]);
  const float cnt = (float)len;
  const float v = len > 0 ? __fdiv_rn(acc, fmaxf(cnt, 1.f)) : zP[((int64_t)h * T + init[i]) * kRC + c];
  cent[((int64_t)h * C + i) * kRC + c] = v;
  if (c == 0) nb[(int64_t)h * C + i] = cnt;
}

// ---------------------------------------------------------------- cluster sums
// one warp per (head, cluster): Sk, Sk2, Sv summed over members in position order (fp32)
__global__ void __launch_bounds__(128) cluster_sums_kernel(const __nv_bfloat16* K, const __nv_bfloat16* V, int Lmax,
                                                           int C, const int32_t* mem, int64_t mem_stride,
                                                           const int32_t* cstart, const int32_t* clen, float* Sk,
                                                           float* Sk2, float* Sv, int nq) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);  // h * C + i
  if (gw >= nq * C) return;
  const int h = gw / C, i = gw % C;
  const int st = cstart[h * C + i], len = clen[h * C + i];
  const int32_t* mp = mem + (int64_t)h * mem_stride + st;
  const __nv_bfloat16* Kh = K + (int64_t)(h / kG) * Lmax * kD;
  const __nv_bfloat16* Vh = V + (int64_t)(h / kG) * Lmax * kD;
  float sk[4] = {0.f, 0.f, 0.f, 0.f}, sk2[4] = {0.f, 0.f, 0.f, 0.f}, sv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < len; ++j) {
    const int t = mp[j];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float kf = __bfloat162float(Kh[(int64_t)t * kD + lane + 32 * u]);
      const float vf = __bfloat162float(Vh[(int64_t)t * kD + lane + 32 * u]);
      sk[u] = __fadd_rn(sk[u], kf);
      sk2[u] = __fadd_rn(sk2[u], __fmul_rn(kf, kf));
      sv[u] = __fadd_rn(sv[u], vf);
    }
  }
  const int64_t o = ((int64_t)h * C + i) * kD;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    Sk[o + lane + 32 * u] = sk[u];
    Sk2[o + lane + 32 * u] = sk2[u];
    Sv[o + lane + 32 * u] = sv[u];
  }
}

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace
}  // namespace oa

using namespace oa;

// hkv (1..8): the KV heads of the request this call builds (a shard of its 8 holds a subset; their query
// heads are the 4 hkv that read them).  Every array argument covers those heads only.
extern "C" int oa_build_codes(const void* K, int64_t hkv, int64_t Lmax, int64_t T, const float* U, float* scale,
                              int8_t* codes, uint32_t* amax_ws, void* stream) {
  const char* fn = "oa_build_codes";
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(T > 0 && T <= Lmax && Lmax < (1ll << 30), "%s: need 0 < T <= Lmax", fn);
  OA_REQUIRE(K && U && scale && codes && amax_ws, "%s: null pointer", fn);
  OA_REQUIRE(oa_aligned16(K) && oa_aligned16(codes), "%s: K and codes must be 16-byte aligned", fn);
  cudaError_t e = cudaMemsetAsync(amax_ws, 0, sizeof(uint32_t) * hkv * kRQ, S(stream));
  if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
  dim3 grid((unsigned)((T + kBT - 1) / kBT), (unsigned)hkv);
  const __nv_bfloat16* Kb = static_cast<const __nv_bfloat16*>(K);
  build_codes_kernel<false><<<grid, kBT, 0, S(stream)>>>(Kb, (int)Lmax, (int)T, U, amax_ws, nullptr, nullptr);
  build_scale_kernel<<<1, kHKV * kRQ, 0, S(stream)>>>(amax_ws, scale, (int)(hkv * kRQ));
  build_codes_kernel<true><<<grid, kBT, 0, S(stream)>>>(Kb, (int)Lmax, (int)T, U, nullptr, scale, codes);
  return oa_check_launch(fn);
}

extern "C" size_t oa_build_project_workspace_bytes(int64_t T) {
  return sizeof(double) * kHQ * kRC * (size_t)((T + kBT - 1) / kBT);
}

extern "C" int oa_build_project(const void* K, int64_t hkv, int64_t Lmax, int64_t T, const void* W, float* zP,
                                float* colmean, void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "oa_build_project";
  OA_REQUIRE_HKV(fn, hkv);
  const int nq = (int)(kG * hkv);
  OA_REQUIRE(T > 0 && T <= Lmax && Lmax < (1ll << 30), "%s: need 0 < T <= Lmax", fn);
  OA_REQUIRE(K && W && zP && colmean && workspace, "%s: null pointer", fn);
  OA_REQUIRE(oa_aligned16(K) && oa_aligned16(workspace), "%s: K and workspace must be 16-byte aligned", fn);
  const int ntiles = (int)((T + kBT - 1) / kBT);
  OA_REQUIRE(workspace_bytes >= oa_build_project_workspace_bytes(T), "%s: workspace too small", fn);
  double* part = static_cast<double*>(workspace);
  project_kernel<<<dim3(ntiles, nq), kBT, 0, S(stream)>>>(static_cast<const __nv_bfloat16*>(K), (int)Lmax, (int)T,
                                                         static_cast<const __nv_bfloat16*>(W), zP, part);
  colmean_kernel<<<1, kHQ * kRC, 0, S(stream)>>>(part, ntiles, (int)T, colmean, nq);
  const int64_t total = (int64_t)nq * T * kRC;
  center_kernel<<<(unsigned)((total + 255) / 256), 256, 0, S(stream)>>>(zP, (int)T, colmean, nq);
  return oa_check_launch(fn);
}

extern "C" int oa_kmeans_assign(const float* zP, int64_t hkv, int64_t T, int64_t C, const float* cent, int32_t* asg,
                                int64_t asg_stride, void* stream) {
  const char* fn = "oa_kmeans_assign";
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(T > 0 && C > 0 && C <= 1024 && asg_stride >= T, "%s: bad sizes", fn);
  OA_REQUIRE(zP && cent && asg && oa_aligned16(zP), "%s: null or misaligned pointer", fn);
  const size_t smem = sizeof(float) * (size_t)C * (kRC + 1);
  if (int rc = oa_smem_opt_in(reinterpret_cast<const void*>(kmeans_assign_kernel), smem, fn)) return rc;
  kmeans_assign_kernel<<<dim3((unsigned)((T + kBT - 1) / kBT), (unsigned)(kG * hkv)), kBT, smem, S(stream)>>>(
      zP, (int)T, (int)C, cent, asg, asg_stride);
  return oa_check_launch(fn);
}

extern "C" size_t oa_csr_workspace_bytes(int64_t T, int64_t C) {
  return sizeof(int32_t) * kHQ * (size_t)C * (size_t)((T + kBT - 1) / kBT);
}

extern "C" int oa_csr_build(const int32_t* asg, int64_t asg_stride, int64_t hkv, int64_t T, int64_t C, int32_t* mem,
                            int64_t mem_stride, int32_t* cstart, int32_t* clen, void* workspace,
                            size_t workspace_bytes, void* stream) {
  const char* fn = "oa_csr_build";
  OA_REQUIRE_HKV(fn, hkv);
  const unsigned nq = (unsigned)(kG * hkv);
  OA_REQUIRE(T > 0 && C > 0 && C <= 1024 && asg_stride >= T && mem_stride >= T, "%s: bad sizes", fn);
  OA_REQUIRE(asg && mem && cstart && clen && workspace, "%s: null pointer", fn);
  OA_REQUIRE(workspace_bytes >= oa_csr_workspace_bytes(T, C), "%s: workspace too small", fn);
  const int ntiles = (int)((T + kBT - 1) / kBT);
  int32_t* tilecnt = static_cast<int32_t*>(workspace);
  csr_count_kernel<<<dim3(ntiles, nq), kBT, sizeof(int) * C, S(stream)>>>(asg, asg_stride, (int)T, (int)C, tilecnt);
  csr_offsets_kernel<<<nq, 256, 0, S(stream)>>>(tilecnt, ntiles, (int)C, cstart, clen);
  csr_place_kernel<<<dim3(ntiles, nq), kBT, 0, S(stream)>>>(asg, asg_stride, (int)T, (int)C, tilecnt, cstart, mem,
                                                           mem_stride);
  return oa_check_launch(fn);
}

extern "C" int oa_kmeans_update(const float* zP, int64_t hkv, int64_t T, int64_t C, const int32_t* mem,
                                int64_t mem_stride, const int32_t* cstart, const int32_t* clen, const int64_t* init,
                                float* cent, float* nb, void* stream) {
  const char* fn = "oa_kmeans_update";
  OA_REQUIRE_HKV(fn, hkv);
  OA_REQUIRE(T > 0 && C > 0 && C <= 1024, "%s: bad sizes", fn);
  OA_REQUIRE(zP && mem && cstart && clen && init && cent && nb, "%s: null pointer", fn);
  kmeans_update_kernel<<<dim3((unsigned)((C * kRC + 127) / 128), (unsigned)(kG * hkv)), 128, 0, S(stream)>>>(
      zP, (int)T, (int)C, mem, mem_stride, cstart, clen, init, cent, nb);
  return oa_check_launch(fn);
}

extern "C" int oa_cluster_sums(const void* K, const void* V, int64_t hkv, int64_t Lmax, int64_t C, const int32_t* mem,
                               int64_t mem_stride, const int32_t* cstart, const int32_t* clen, float* Sk, float* Sk2,
                               float* Sv, void* stream) {
  const char* fn = "oa_cluster_sums";
  OA_REQUIRE_HKV(fn, hkv);
  const int nq = (int)(kG * hkv);
  OA_REQUIRE(Lmax > 0 && C > 0 && C <= 1024, "%s: bad sizes", fn);
  OA_REQUIRE(K && V && mem && cstart && clen && Sk && Sk2 && Sv, "%s: null pointer", fn);
  cluster_sums_kernel<<<(unsigned)((nq * C + 3) / 4), 128, 0, S(stream)>>>(
      static_cast<const __nv_bfloat16*>(K), static_cast<const __nv_bfloat16*>(V), (int)Lmax, (int)C, mem, mem_stride,
      cstart, clen, Sk, Sk2, Sv, nq);
  return oa_check_launch(fn);
}
