// OpenAttention.flash on sm_100a: one online softmax per query row over the selected tokens (S),
// the expanded tokens (X) and the count-aware cluster proxies (P).
//
// Semantics follow _decode_expand_kernel (triton_expand_decode.py:31-136) and _ours_flash_kernel
// (inference/methods_eager.py:91-158): token logit q.k*s, proxy logit q.kbar*s + ln n, both in the
// log2 domain; pads (-1) and -inf proxies are skipped; an empty row yields zeros.  The split-K mode
// replaces _k_ours_flash_split + _k_dense_combine (inference/ours_graph.py:214-262,
// inference/graph_runner.py:299-312): partial (m, l, acc) per chunk, merged with weights 2^(m - max).
//
// Design: one CTA (4 warps) per (row, chunk).  Each half-warp owns one list entry at a time: 16
// lanes x 16 B cover the 256-byte bf16 K row and the V row, so every gathered row is one fully used
// 256-byte burst.  Each half-warp keeps UNROLL entries (K and V) in flight before it reduces, and
// keeps its own online-softmax state; the 8 half-warp states are merged through shared memory.
// Proxy rows whose ln n is -inf are never read.  In split mode the last CTA of a row to finish
// (atomic ticket, no waiting) merges the row's partials in chunk order, so the result does not
// depend on which CTA finishes last.
#include "oa_common.cuh"

#include <mutex>
#include "../../include/openattention_b200.h"

namespace oa {
namespace {

constexpr int kUnroll = 4;
constexpr int kThreads = 128;
constexpr int kHalfWarps = kThreads / 16;

struct FlashArgs {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t kv_sh, kv_st;
  const int32_t* sel;
  const int32_t* exp;
  int n_sel, n_exp;
  const __nv_bfloat16* kbar;
  const __nv_bfloat16* vbar;
  int64_t kb_sh, kb_sb;
  const float* logn;
  int64_t ln_stride;
  void* out;
  int64_t out_stride;
  int G;
  int64_t K;
  int NB;
  float qk_scale;  // sm_scale * log2(e)
  int nsplit, chunk;
  float* pm;
  float* pl;
  float* pacc;
  unsigned* cnt;
};

__device__ __forceinline__ void unpack8(const uint4& w, float* f) {
  f[0] = bf_lo(w.x); f[1] = bf_hi(w.x); f[2] = bf_lo(w.y); f[3] = bf_hi(w.y);
  f[4] = bf_lo(w.z); f[5] = bf_hi(w.z); f[6] = bf_lo(w.w); f[7] = bf_hi(w.w);
}

template <bool QHEAD, bool OUTF32>
__global__ void __launch_bounds__(kThreads) flash_kernel(const FlashArgs a) {
  const int r = blockIdx.x;
  const int split = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int hw = (tid >> 5) * 2 + (lane >> 4);  // half-warp 0..7
  const int hl = lane & 15;                     // dims hl*8 .. hl*8+7
  const int kvh = r / a.G;
  const int64_t prow = QHEAD ? (int64_t)r : (int64_t)kvh;
  const __nv_bfloat16* Kr = a.k + (int64_t)kvh * a.kv_sh;
  const __nv_bfloat16* Vr = a.v + (int64_t)kvh * a.kv_sh;

  float qf[8];
  unpack8(*reinterpret_cast<const uint4*>(a.q + (int64_t)r * a.q_stride + hl * 8), qf);

  const int nse = a.n_sel + a.n_exp;
  const int total = nse + a.NB;
  const int start = split * a.chunk;
  const int end = min(start + a.chunk, total);

  float m = -INFINITY, l = 0.f;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;

  for (int base = start; base < end; base += kHalfWarps * kUnroll) {
    uint4 kw[kUnroll], vw[kUnroll];
    float bias[kUnroll];
    bool ok[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = base + hw + kHalfWarps * u;
      ok[u] = false;
      bias[u] = 0.f;
      const __nv_bfloat16* kp = nullptr;
      const __nv_bfloat16* vp = nullptr;
      if (j < end) {
        if (j < nse) {
          const int t = j < a.n_sel ? a.sel[(int64_t)r * a.n_sel + j]
                                    : a.exp[(int64_t)r * a.n_exp + (j - a.n_sel)];
          if (t >= 0 && (int64_t)t < a.K) {
            ok[u] = true;
            kp = Kr + (int64_t)t * a.kv_st;
            vp = Vr + (int64_t)t * a.kv_st;
          }
        } else {
          const int b = j - nse;
          const float ln = a.logn[(int64_t)r * a.ln_stride + b];
          if (ln > -INFINITY) {
            ok[u] = true;
            bias[u] = ln * kLog2e;
            kp = a.kbar + prow * a.kb_sh + (int64_t)b * a.kb_sb;
            vp = a.vbar + prow * a.kb_sh + (int64_t)b * a.kb_sb;
          }
        }
      }
      if (ok[u]) {
        kw[u] = ldg_stream(kp + hl * 8);
        vw[u] = ldg_stream(vp + hl * 8);
      } else {
        kw[u] = make_uint4(0u, 0u, 0u, 0u);
        vw[u] = kw[u];
      }
    }
    float z[kUnroll];
    float mx = m;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float kf[8];
      unpack8(kw[u], kf);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qf[i], kf[i], d);
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      z[u] = ok[u] ? fmaf(d, a.qk_scale, bias[u]) : -INFINITY;
      mx = fmaxf(mx, z[u]);
    }
    if (mx == -INFINITY) continue;
    const float alpha = exp2f(m - mx);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= alpha;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const float p = exp2f(z[u] - mx);
      float vf[8];
      unpack8(vw[u], vf);
      l += p;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(p, vf[i], acc[i]);
    }
    m = mx;
  }

  __shared__ float s_m[kHalfWarps], s_l[kHalfWarps];
  __shared__ float s_acc[kHalfWarps][kD];
  __shared__ unsigned s_last;
  if (hl == 0) {
    s_m[hw] = m;
    s_l[hw] = l;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) s_acc[hw][hl * 8 + i] = acc[i];
  __syncthreads();

  float M = -INFINITY;
#pragma unroll
  for (int h = 0; h < kHalfWarps; ++h) M = fmaxf(M, s_m[h]);
  float L = 0.f, A = 0.f;
  if (M > -INFINITY) {
#pragma unroll
    for (int h = 0; h < kHalfWarps; ++h) {
      const float w = exp2f(s_m[h] - M);
      L = fmaf(w, s_l[h], L);
      A = fmaf(w, s_acc[h][tid], A);
    }
  }

  auto store = [&](float val) {
    if (OUTF32)
      reinterpret_cast<float*>(a.out)[(int64_t)r * a.out_stride + tid] = val;
    else
      reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)r * a.out_stride + tid] = __float2bfloat16_rn(val);
  };

  if (a.nsplit == 1) {
    store(L > 0.f ? A / L : 0.f);
    return;
  }
  const int64_t pi = (int64_t)r * a.nsplit + split;
  a.pacc[pi * kD + tid] = A;
  if (tid == 0) {
    a.pm[pi] = M;
    a.pl[pi] = L;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&a.cnt[r], 1u) == (unsigned)(a.nsplit - 1)) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t p0 = (int64_t)r * a.nsplit;
  float MM = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) MM = fmaxf(MM, __ldcg(&a.pm[p0 + s]));
  float LL = 0.f, AA = 0.f;
  if (MM > -INFINITY) {
    for (int s = 0; s < a.nsplit; ++s) {
      const float w = exp2f(__ldcg(&a.pm[p0 + s]) - MM);
      LL = fmaf(w, __ldcg(&a.pl[p0 + s]), LL);
      AA = fmaf(w, __ldcg(&a.pacc[(p0 + s) * kD + tid]), AA);
    }
  }
  store(LL > 0.f ? AA / LL : 0.f);
  if (tid == 0) a.cnt[r] = 0u;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int resolve_split(int64_t BQ, int64_t total, int nsplit, int* chunk_out) {
  int ns = nsplit;
  if (ns <= 0) {
    ns = BQ >= 512 ? 1 : (int)std::min<int64_t>(32, (4 * 148 + BQ - 1) / BQ);
    ns = (int)std::min<int64_t>(ns, std::max<int64_t>(1, (total + 15) / 16));
  }
  ns = std::max(1, std::min(ns, 64));
  ns = (int)std::min<int64_t>(ns, std::max<int64_t>(1, (total + 7) / 8));
  int64_t chunk = (total + ns - 1) / ns;
  chunk = (chunk + 7) & ~int64_t(7);
  if (chunk <= 0) chunk = 8;
  ns = (int)std::max<int64_t>(1, (total + chunk - 1) / chunk);
  *chunk_out = (int)chunk;
  return ns;
}

size_t workspace_bytes(int64_t BQ, int ns) {
  if (ns <= 1) return 0;
  const size_t parts = (size_t)BQ * (size_t)ns;
  return 2 * align256(parts * sizeof(float)) + align256(parts * kD * sizeof(float)) +
         align256((size_t)BQ * sizeof(unsigned));
}

int flash_entry(bool qhead, const void* q, int64_t q_stride, const void* k, const void* v, int64_t kv_sh,
                int64_t kv_st, const int32_t* sel, int64_t n_sel, const int32_t* exp_idx, int64_t n_exp,
                const void* kbar, const void* vbar, int64_t kb_sh, int64_t kb_sb, const float* log_n,
                int64_t ln_stride, void* out, int64_t out_stride, int out_dtype, int64_t BQ, int64_t BH,
                int64_t K, int64_t NB, float sm_scale, int nsplit, void* workspace, size_t ws_bytes,
                void* stream, const char* fn_name = nullptr, bool clear_tickets = false) {
  // fn_name: the entry point named in error messages; clear_tickets: zero the split's ticket counters on
  // `stream` before the kernel, once every argument has been checked (a rejected call changes nothing)
  const char* fn = fn_name ? fn_name : (qhead ? "oa_flash_qhead_proxies" : "oa_flash_kvhead_proxies");
  OA_REQUIRE(BQ > 0 && BH > 0 && BQ % BH == 0, "%s: need BQ > 0, BH > 0 and BQ %% BH == 0 (BQ=%lld BH=%lld)",
             fn, (long long)BQ, (long long)BH);
  OA_REQUIRE(BQ <= 0x7fffffff, "%s: BQ too large", fn);
  OA_REQUIRE(n_sel >= 0 && n_exp >= 0 && NB >= 0 && K >= 0, "%s: negative size", fn);
  OA_REQUIRE(n_sel + n_exp + NB < (int64_t)1 << 30, "%s: index list too long", fn);
  OA_REQUIRE(q && k && v && out, "%s: null q/k/v/out", fn);
  OA_REQUIRE(n_sel == 0 || sel, "%s: null sel_idx", fn);
  OA_REQUIRE(n_exp == 0 || exp_idx, "%s: null exp_idx", fn);
  OA_REQUIRE(NB == 0 || (kbar && vbar && log_n), "%s: null kbar/vbar/log_n with NB > 0", fn);
  OA_REQUIRE(out_dtype == OA_BF16 || out_dtype == OA_F32, "%s: out_dtype must be OA_BF16 or OA_F32", fn);
  OA_REQUIRE(oa_aligned16(q) && oa_aligned16(k) && oa_aligned16(v), "%s: q/k/v must be 16-byte aligned", fn);
  OA_REQUIRE(q_stride % 8 == 0 && kv_sh % 8 == 0 && kv_st % 8 == 0,
             "%s: q and k/v strides must be multiples of 8 elements (16 bytes)", fn);
  if (NB > 0) {
    OA_REQUIRE(oa_aligned16(kbar) && oa_aligned16(vbar), "%s: kbar/vbar must be 16-byte aligned", fn);
    OA_REQUIRE(kb_sh % 8 == 0 && kb_sb % 8 == 0, "%s: kbar/vbar strides must be multiples of 8 elements",
               fn);
  }
  const int64_t total = n_sel + n_exp + NB;
  int chunk = 8;
  const int ns = resolve_split(BQ, total, nsplit, &chunk);
  FlashArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.kv_sh = kv_sh;
  a.kv_st = kv_st;
  a.sel = sel;
  a.exp = exp_idx;
  a.n_sel = (int)n_sel;
  a.n_exp = (int)n_exp;
  a.kbar = static_cast<const __nv_bfloat16*>(kbar);
  a.vbar = static_cast<const __nv_bfloat16*>(vbar);
  a.kb_sh = kb_sh;
  a.kb_sb = kb_sb;
  a.logn = log_n;
  a.ln_stride = ln_stride;
  a.out = out;
  a.out_stride = out_stride;
  a.G = (int)(BQ / BH);
  a.K = K;
  a.NB = (int)NB;
  a.qk_scale = sm_scale * kLog2e;
  a.nsplit = ns;
  a.chunk = chunk;
  a.pm = a.pl = a.pacc = nullptr;
  a.cnt = nullptr;
  if (ns > 1) {
    const size_t need = workspace_bytes(BQ, ns);
    OA_REQUIRE(workspace && ws_bytes >= need && oa_aligned16(workspace),
               "%s: split into %d chunks needs a 16-byte aligned workspace of %zu bytes (got %zu)", fn, ns,
               need, ws_bytes);
    // ticket counters first (their place depends on BQ only), then the partial (m, l, acc) arrays
    const size_t parts = (size_t)BQ * ns;
    char* w = static_cast<char*>(workspace);
    a.cnt = reinterpret_cast<unsigned*>(w);
    w += align256((size_t)BQ * sizeof(unsigned));
    a.pm = reinterpret_cast<float*>(w);
    a.pl = reinterpret_cast<float*>(w + align256(parts * sizeof(float)));
    a.pacc = reinterpret_cast<float*>(w + 2 * align256(parts * sizeof(float)));
  }
  dim3 grid((unsigned)BQ, (unsigned)ns);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (clear_tickets && a.cnt != nullptr) {
    const cudaError_t e = cudaMemsetAsync(a.cnt, 0, (size_t)BQ * sizeof(unsigned), st);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: clearing the ticket counters failed: %s", fn, cudaGetErrorString(e));
  }
  if (qhead) {
    if (out_dtype == OA_F32)
      flash_kernel<true, true><<<grid, kThreads, 0, st>>>(a);
    else
      flash_kernel<true, false><<<grid, kThreads, 0, st>>>(a);
  } else {
    if (out_dtype == OA_F32)
      flash_kernel<false, true><<<grid, kThreads, 0, st>>>(a);
    else
      flash_kernel<false, false><<<grid, kThreads, 0, st>>>(a);
  }
  return oa_check_launch(fn);
}

}  // namespace
}  // namespace oa

extern "C" size_t oa_flash_workspace_bytes(int64_t BQ, int64_t n_sel, int64_t n_exp, int64_t NB, int nsplit) {
  int chunk = 8;
  const int ns = oa::resolve_split(BQ, n_sel + n_exp + NB, nsplit, &chunk);
  return oa::workspace_bytes(BQ, ns);
}

extern "C" int oa_flash_kvhead_proxies(const void* q, int64_t q_stride, const void* k, const void* v,
                                       int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel,
                                       int64_t n_sel, const int32_t* exp_idx, int64_t n_exp, const void* kbar,
                                       const void* vbar, int64_t kbar_stride_h, int64_t kbar_stride_b,
                                       const float* log_n, int64_t log_n_stride, void* out, int64_t out_stride,
                                       int out_dtype, int64_t BQ, int64_t BH, int64_t K, int64_t NB,
                                       float sm_scale, int nsplit, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  return oa::flash_entry(false, q, q_stride, k, v, kv_stride_h, kv_stride_t, sel, n_sel, exp_idx, n_exp, kbar,
                         vbar, kbar_stride_h, kbar_stride_b, log_n, log_n_stride, out, out_stride, out_dtype, BQ,
                         BH, K, NB, sm_scale, nsplit, workspace, workspace_bytes, stream);
}

extern "C" int oa_flash_qhead_proxies(const void* q, int64_t q_stride, const void* k, const void* v,
                                      int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel, int64_t n_sel,
                                      const int32_t* exp_idx, int64_t n_exp, const void* kbar, const void* vbar,
                                      int64_t kbar_stride_h, int64_t kbar_stride_b, const float* log_n,
                                      int64_t log_n_stride, void* out, int64_t out_stride, int out_dtype,
                                      int64_t BQ, int64_t BH, int64_t K, int64_t NB, float sm_scale, int nsplit,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  return oa::flash_entry(true, q, q_stride, k, v, kv_stride_h, kv_stride_t, sel, n_sel, exp_idx, n_exp, kbar,
                         vbar, kbar_stride_h, kbar_stride_b, log_n, log_n_stride, out, out_stride, out_dtype, BQ,
                         BH, K, NB, sm_scale, nsplit, workspace, workspace_bytes, stream);
}

// ------------------------------------------------------------------------------------------------
// Split-K flash without caller-provided workspace.  Some callers cannot call cudaMalloc: a plugin
// handed only raw device pointers across a foreign-function boundary (no allocator of its own), a
// serving host that has already given all device memory to its own pool, or a decode loop that
// must not let an allocation stall the device.  For them the split-K scratch (ticket counters and
// the partial (m, l, acc) arrays) lives in one fixed file-scope array that every GPU loading this
// library holds until the process exits.
namespace oa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kNoAllocMaxDevices = 64;

__device__ __align__(256) unsigned char g_flash_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kNoAllocMaxDevices] = {};

// Device address of g_flash_scratch on the current device, looked up once per device (with that
// device current) and kept for later calls.  Returns a status; *out is set on success.  The kept
// address belongs to the device's primary context: after cudaDeviceReset (or anything else that
// destroys and recreates that context) it is stale, and this entry point must not be used again in
// the process.
int scratch_on_current_device(const char* fn, void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: cudaGetDevice failed: %s", fn, cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return oa_fail(OA_ERR_UNSUPPORTED, "%s: device ordinal %d is beyond the %d devices this entry point tracks", fn,
                   dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_flash_scratch);
    if (e != cudaSuccess || !p)
      return oa_fail(OA_ERR_CUDA, "%s: cudaGetSymbolAddress of the scratch array failed on device %d: %s", fn, dev,
                     cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return OA_OK;
}

}  // namespace
}  // namespace oa

extern "C" int oa_flash_qhead_proxies_noalloc(const void* q, int64_t q_stride, const void* k, const void* v,
                                              int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel,
                                              int64_t n_sel, const int32_t* exp_idx, int64_t n_exp,
                                              const void* kbar, const void* vbar, int64_t kbar_stride_h,
                                              int64_t kbar_stride_b, const float* log_n, int64_t log_n_stride,
                                              void* out, int64_t out_stride, int out_dtype, int64_t BQ,
                                              int64_t BH, int64_t K, int64_t NB, float sm_scale, int nsplit,
                                              void* stream) {
  const char* fn = "oa_flash_qhead_proxies_noalloc";
  OA_REQUIRE(BQ > 0 && BQ <= 0x7fffffff && n_sel >= 0 && n_exp >= 0 && NB >= 0 &&
                 n_sel + n_exp + NB < (int64_t)1 << 30,
             "%s: bad sizes (BQ=%lld n_sel=%lld n_exp=%lld NB=%lld)", fn, (long long)BQ, (long long)n_sel,
             (long long)n_exp, (long long)NB);
  int chunk = 8;
  const int ns = oa::resolve_split(BQ, n_sel + n_exp + NB, nsplit, &chunk);
  const size_t need = oa::workspace_bytes(BQ, ns);
  OA_REQUIRE(need <= oa::kNoAllocScratchBytes,
             "%s: %d chunks for %lld rows need %zu bytes of scratch, above this entry point's fixed %zu bytes; "
             "pass a smaller nsplit or use oa_flash_qhead_proxies with a workspace",
             fn, ns, (long long)BQ, need, oa::kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = oa::scratch_on_current_device(fn, &scratch);
    if (rc != OA_OK) return rc;
  }
  // The ticket counters must start at zero: flash_entry clears them on the stream (rather than trust what
  // an earlier call left), after it has checked every argument, so a rejected call leaves the array as it was.
  return oa::flash_entry(true, q, q_stride, k, v, kv_stride_h, kv_stride_t, sel, n_sel, exp_idx, n_exp, kbar,
                         vbar, kbar_stride_h, kbar_stride_b, log_n, log_n_stride, out, out_stride, out_dtype, BQ,
                         BH, K, NB, sm_scale, nsplit, scratch, need, stream, fn, /*clear_tickets=*/true);
}
