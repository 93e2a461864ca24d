// Router (logits + softmax + top-k), expert alignment, permute and combine.
//
// Routing restates RouterCapture's recomputation of the external block's
// router (src/LLaDA_Quant/trajectory/llada.py:225-234):
//   logits = bf16(x . gate_w^T)   fp32 accumulation, one rounding
//   p      = softmax(logits (+ bias), fp32)  = exp(l - max) * (1 / sum)
//   top-k  larger p first; equal p -> smaller expert id (torch's CPU topk
//          leaves that order unspecified)
// Alignment groups the T*k (token, slot) entries by expert, stable in entry
// order (the contract of the external moe_align_block_size,
// INFERENCE_REPO_CHANGES.md:274-278).
#include <cstdlib>

#include "llq_common.cuh"
#include "ep_window.cuh"

namespace llq {

namespace {

constexpr int kMaxExperts = 256;

// softmax + top-k of one token held by one warp: value j of the lane is
// expert lane + 32 j (J values per lane: E <= 32 J)
template <int J = kMaxExperts / 32>
__device__ void warp_softmax_topk(float (&v)[kMaxExperts / 32], int E, int k, int renormalize,
                                  float* __restrict__ topk_w, int32_t* __restrict__ topk_ids) {
  const int lane = threadIdx.x & 31;
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < J; ++j)
    if (lane + 32 * j < E) m = fmaxf(m, v[j]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    if (lane + 32 * j < E) {
      v[j] = expf(__fsub_rn(v[j], m));
      s = __fadd_rn(s, v[j]);
    }
  }
  s = warp_sum(s);
  const float inv = __fdiv_rn(1.f, s);
#pragma unroll
  for (int j = 0; j < J; ++j) v[j] = (lane + 32 * j < E) ? __fmul_rn(v[j], inv) : -1.f;

  float wsum = 0.f;
  float chosen_w = 0.f;
  int chosen_id = 0;
  for (int r = 0; r < k; ++r) {
    // (value desc, id asc): the probabilities are >= +0 and the taken ones -2, so
    // their bit patterns order like the values as signed integers; one warp max
    // of the bits, then the smallest id holding it
    int bb = static_cast<int>(0x80000000u);
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int id = lane + 32 * j;
      const int b = __float_as_int(v[j]);
      if (id < E && b > bb) {  // ids ascend with j: the first of equal values is kept
        bb = b;
        bi = id;
      }
    }
    const int wb = __reduce_max_sync(0xffffffffu, bb);
    bi = __reduce_min_sync(0xffffffffu, bb == wb ? bi : 0x7fffffff);
    const float bv = __int_as_float(wb);
    // remove the winner
#pragma unroll
    for (int j = 0; j < J; ++j)
      if (lane + 32 * j == bi) v[j] = -2.f;
    if (lane == r) {
      chosen_w = bv;
      chosen_id = bi;
    }
    wsum = __fadd_rn(wsum, bv);
  }
  if (lane < k) {
    topk_ids[lane] = chosen_id;
    topk_w[lane] = renormalize ? __fdiv_rn(chosen_w, wsum) : chosen_w;
  }
}

// logits + softmax + top-k for TOK tokens per block of 256 threads.  Token
// rows are staged in shared memory as fp32; each warp owns experts
// warp, warp + 8, ...; lane l sums the 16-byte weight vectors l, l + 32, ...
// of an expert (every load of a pass issued before any is consumed), then a
// butterfly sum -- the same order for every TOK, so the logits do not depend
// on how tokens are grouped into blocks.
constexpr int kRouteThreads = 256;

template <int TOK>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const __nv_bfloat16* __restrict__ gate_w,
                                                              int64_t T, int H, int E, int k,
                                                              const float* __restrict__ bias, int renormalize,
                                                              __nv_bfloat16* __restrict__ logits_out,
                                                              float* __restrict__ topk_w,
                                                              int32_t* __restrict__ topk_ids) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);                        // [TOK][H]
  float* lg = xs + TOK * static_cast<int64_t>(H);                        // [TOK][E]
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * TOK;
  const int nt = static_cast<int>(T - t0 < TOK ? T - t0 : TOK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = kRouteThreads / 32;

  const int vec_per_row = H / 8;
  for (int i = threadIdx.x; i < TOK * vec_per_row; i += blockDim.x) {
    const int t = i / vec_per_row, v = i - t * vec_per_row;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (t < nt) val = __ldg(reinterpret_cast<const uint4*>(x + (t0 + t) * H) + v);
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(&val);
    float4 lo, hi;
    lo.x = __bfloat162float(p[0]); lo.y = __bfloat162float(p[1]);
    lo.z = __bfloat162float(p[2]); lo.w = __bfloat162float(p[3]);
    hi.x = __bfloat162float(p[4]); hi.y = __bfloat162float(p[5]);
    hi.z = __bfloat162float(p[6]); hi.w = __bfloat162float(p[7]);
    float4* dst = reinterpret_cast<float4*>(xs + static_cast<int64_t>(t) * H) + 2 * v;
    dst[0] = lo;
    dst[1] = hi;
  }
  __syncthreads();

  constexpr int U = 8;  // vectors per lane per pass (H = 2048 -> one pass)
  for (int e0 = warp; e0 < E; e0 += 2 * NW) {
    const int e1 = e0 + NW;
    float acc0[TOK], acc1[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc0[t] = acc1[t] = 0.f;
    const uint4* w0 = reinterpret_cast<const uint4*>(gate_w + static_cast<int64_t>(e0) * H);
    const uint4* w1 = reinterpret_cast<const uint4*>(gate_w + static_cast<int64_t>(e1 < E ? e1 : e0) * H);
    for (int vb = 0; vb < vec_per_row; vb += 32 * U) {
      uint4 a[U], b[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = vb + lane + 32 * u;
        a[u] = v < vec_per_row ? __ldg(w0 + v) : make_uint4(0, 0, 0, 0);
        b[u] = (v < vec_per_row && e1 < E) ? __ldg(w1 + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = vb + lane + 32 * u;
        if (v >= vec_per_row) break;
        const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&a[u]);
        const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&b[u]);
        float wa[8], wb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          wa[i] = __bfloat162float(ap[i]);
          wb[i] = __bfloat162float(bp[i]);
        }
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
          const float4* xv = reinterpret_cast<const float4*>(xs + static_cast<int64_t>(t) * H) + 2 * v;
          const float4 x0 = xv[0], x1 = xv[1];
          const float xf[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc0[t] = __fmaf_rn(xf[i], wa[i], acc0[t]);
            acc1[t] = __fmaf_rn(xf[i], wb[i], acc1[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
      const float l0 = round_bf16(warp_sum(acc0[t]));
      const float l1 = round_bf16(warp_sum(acc1[t]));
      if (lane == 0) {
        lg[t * E + e0] = l0;
        if (e1 < E) lg[t * E + e1] = l1;
      }
    }
  }
  __syncthreads();

  for (int tw = warp; tw < nt; tw += NW) {
    const int64_t t = t0 + tw;
    float v[kMaxExperts / 32];
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      const int id = lane + 32 * j;
      float l = 0.f;
      if (id < E) {
        l = lg[tw * E + id];
        if (logits_out != nullptr) logits_out[t * E + id] = __float2bfloat16_rn(l);
        if (bias != nullptr) l = __fadd_rn(l, bias[id]);
      }
      v[j] = l;
    }
    warp_softmax_topk(v, E, k, renormalize, topk_w + t * k, topk_ids + t * k);
  }
}

// Router on the tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate):
// 16 tokens x all E experts per block; the 16 warps split H into equal
// slices, and the slices' partial logits are summed in warp order (a fixed
// order, so the result is deterministic).  Within a 32-wide K chunk lane c of
// a quad takes the contiguous elements 8c..8c+7 of both the token row and the
// weight row, so every MMA pairs equal K indices.  Needs E % 8 == 0, E <= 64,
// H % 512 == 0.
constexpr int kRmWarps = 16;

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int NT>
__global__ void __launch_bounds__(kRmWarps * 32) route_mma_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  const __nv_bfloat16* __restrict__ gate_w,
                                                                  int64_t T, int H, int k,
                                                                  const float* __restrict__ bias, int renormalize,
                                                                  __nv_bfloat16* __restrict__ logits_out,
                                                                  float* __restrict__ topk_w,
                                                                  int32_t* __restrict__ topk_ids) {
  constexpr int E = NT * 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* part = reinterpret_cast<float*>(smem_raw);  // [warp][16 tokens][E]
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int slice = H / kRmWarps;
  const int kbeg = warp * slice;
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const bool r0 = t0 + g < T, r1 = t0 + g + 8 < T;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  const uint4* xa = reinterpret_cast<const uint4*>(x + (t0 + g) * H + kbeg) + c;
  const uint4* xb = reinterpret_cast<const uint4*>(x + (t0 + g + 8) * H + kbeg) + c;
  const uint4* wrow = reinterpret_cast<const uint4*>(gate_w + static_cast<int64_t>(g) * H + kbeg) + c;
  const int64_t nstride = static_cast<int64_t>(8) * H / 8;  // uint4 per 8 weight rows
#pragma unroll 2
  for (int kc = 0; kc < slice; kc += 32) {
    const int q = kc / 8;
    const uint4 a_lo = r0 ? __ldg(xa + q) : zero;
    const uint4 a_hi = r1 ? __ldg(xb + q) : zero;
    uint4 b[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) b[n] = __ldg(wrow + n * nstride + q);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      mma_bf16_16816(acc[n], a_lo.x, a_hi.x, a_lo.y, a_hi.y, b[n].x, b[n].y);
      mma_bf16_16816(acc[n], a_lo.z, a_hi.z, a_lo.w, a_hi.w, b[n].z, b[n].w);
    }
  }
  float* pw = part + warp * 16 * E;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    pw[g * E + n * 8 + 2 * c] = acc[n][0];
    pw[g * E + n * 8 + 2 * c + 1] = acc[n][1];
    pw[(g + 8) * E + n * 8 + 2 * c] = acc[n][2];
    pw[(g + 8) * E + n * 8 + 2 * c + 1] = acc[n][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * E; i += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kRmWarps; ++w) sum = __fadd_rn(sum, part[w * 16 * E + i]);
    part[i] = round_bf16(sum);  // warp 0's slice is read above before this write (same thread, same i)
  }
  __syncthreads();
  pdl_trigger();
  const int nt = static_cast<int>(T - t0 < 16 ? T - t0 : 16);
  if (warp < nt) {
    const int64_t t = t0 + warp;
    float v[kMaxExperts / 32];
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      const int id = lane + 32 * j;
      float l = 0.f;
      if (id < E) {
        l = part[warp * E + id];
        if (logits_out != nullptr) logits_out[t * E + id] = __float2bfloat16_rn(l);
        if (bias != nullptr) l = __fadd_rn(l, bias[id]);
      }
      v[j] = l;
    }
    warp_softmax_topk<(E + 31) / 32>(v, E, k, renormalize, topk_w + t * k, topk_ids + t * k);
  }
}

template <typename L>
__global__ void route_topk_kernel(const L* __restrict__ logits, int64_t T, int E, int k,
                                  const float* __restrict__ bias, int renormalize,
                                  float* __restrict__ topk_w, int32_t* __restrict__ topk_ids) {
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  float v[kMaxExperts / 32];
#pragma unroll
  for (int j = 0; j < kMaxExperts / 32; ++j) {
    const int id = lane + 32 * j;
    float l = 0.f;
    if (id < E) {
      l = to_f32<L>(logits[t * E + id]);
      if (bias != nullptr) l = __fadd_rn(l, bias[id]);
    }
    v[j] = l;
  }
  warp_softmax_topk(v, E, k, renormalize, topk_w + t * k, topk_ids + t * k);
}

// ---------------------------------------------------------------------------
// alignment: count -> scan -> stable scatter
// ---------------------------------------------------------------------------

__device__ __forceinline__ int mask_count(const AlignMask& m, int r) {
  const int c = static_cast<int>(ld_acquire_sys(m.counts + r));
  return c < m.cap ? (c < 0 ? 0 : c) : m.cap;
}

constexpr int kAlignChunk = 2048;  // (token, slot) entries per block
constexpr int kAlignThreads = 256;

__global__ void __launch_bounds__(kAlignThreads) align_count_kernel(
    const int32_t* __restrict__ ids, int64_t n, int E, int32_t* __restrict__ counts, AlignMask m) {
  __shared__ int32_t c[kMaxExperts];
  __shared__ int32_t vc[kMaxRanks];
  for (int e = threadIdx.x; e < E; e += blockDim.x) c[e] = 0;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < m.clear_n; i += blockDim.x) m.clear[i] = 0;
  if (m.counts != nullptr)
    for (int r = threadIdx.x; r < m.R; r += blockDim.x) vc[r] = mask_count(m, r);
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kAlignChunk;
  const int64_t hi = lo + kAlignChunk < n ? lo + kAlignChunk : n;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    if (m.counts != nullptr && (i % m.cap) >= vc[i / m.cap]) continue;
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&c[e], 1);
    else atomicExch(&g_device_error, 2);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[static_cast<int64_t>(blockIdx.x) * E + e] = c[e];
}

__global__ void __launch_bounds__(kMaxExperts) align_scan_kernel(int32_t* __restrict__ counts,
                                                                 int nblk, int E,
                                                                 int32_t* __restrict__ offsets) {
  __shared__ int32_t tot[kMaxExperts + 1];
  const int e = threadIdx.x;
  int running = 0;
  if (e < E) {
    for (int b = 0; b < nblk; ++b) {
      const int c = counts[static_cast<int64_t>(b) * E + e];
      counts[static_cast<int64_t>(b) * E + e] = running;  // block base, relative to the expert
      running += c;
    }
    tot[e] = running;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      const int c = tot[i];
      tot[i] = acc;
      acc += c;
    }
    tot[E] = acc;
  }
  __syncthreads();
  if (e < E) {
    offsets[e] = tot[e];
    for (int b = 0; b < nblk; ++b) counts[static_cast<int64_t>(b) * E + e] += tot[e];
  }
  if (e == 0) offsets[E] = tot[E];
}

__global__ void __launch_bounds__(kAlignThreads) align_scatter_kernel(
    const int32_t* __restrict__ ids, int64_t n, int E, const int32_t* __restrict__ base,
    int32_t* __restrict__ sorted_slots, AlignMask m) {
  __shared__ int32_t cursor[kMaxExperts];
  __shared__ int32_t vc[kMaxRanks];
  if (m.counts != nullptr)
    for (int r = threadIdx.x; r < m.R; r += blockDim.x) vc[r] = mask_count(m, r);
  __shared__ int32_t wcnt[kAlignThreads / 32][kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = base[static_cast<int64_t>(blockIdx.x) * E + e];
  for (int i = threadIdx.x; i < (kAlignThreads / 32) * kMaxExperts; i += blockDim.x)
    (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kAlignChunk;
  const int64_t hi = lo + kAlignChunk < n ? lo + kAlignChunk : n;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t r0 = lo; r0 < hi; r0 += kAlignThreads) {
    const int64_t i = r0 + threadIdx.x;
    int e = -1;
    if (i < hi && (m.counts == nullptr || (i % m.cap) < vc[i / m.cap])) {
      e = ids[i];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & lt_mask);
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    int pos = 0;
    if (e >= 0) {
      pos = cursor[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w][e];
      sorted_slots[pos] = static_cast<int32_t>(i);
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kAlignThreads / 32; ++w) {
        add += wcnt[w][ee];
        wcnt[w][ee] = 0;
      }
      cursor[ee] += add;
    }
    __syncthreads();
  }
}

// kperm: reorder each 8-element block as [0,4,1,5,2,6,3,7], the K order in
// which the fast-mode expert GEMM lays out its integer weight codes
// Small problems (the decode regime): count, scan and stable scatter in one
// block of 1024 threads, one launch instead of three.
constexpr int kAlignSmallMax = 16384;
constexpr int kAlignSmallThreads = 1024;

__global__ void __launch_bounds__(kAlignSmallThreads) align_small_kernel(
    const int32_t* __restrict__ ids, int n, int E, int32_t* __restrict__ offsets,
    int32_t* __restrict__ sorted_slots, AlignMask m) {
  constexpr int W = kAlignSmallThreads / 32;
  __shared__ int32_t cnt[kMaxExperts];
  __shared__ int32_t vc[kMaxRanks];
  __shared__ int32_t cursor[kMaxExperts];
  __shared__ int32_t wcnt[W][kMaxExperts];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  for (int i = tid; i < m.clear_n; i += blockDim.x) m.clear[i] = 0;
  for (int i = tid; i < kMaxExperts; i += blockDim.x) cnt[i] = 0;
  for (int i = tid; i < W * kMaxExperts; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  if (m.counts != nullptr) {
    if (tid == 0 && m.flags != nullptr) ep_wait_flags(m.flags, m.R, m.epoch, m.timeout_ns, 0x501);
    __syncthreads();
    for (int r = tid; r < m.R; r += blockDim.x) vc[r] = mask_count(m, r);
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    if (m.counts != nullptr && (i % m.cap) >= vc[i / m.cap]) continue;
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else atomicExch(&g_device_error, 2);
  }
  __syncthreads();
  if (warp == 0) {
    constexpr int J = kMaxExperts / 32;
    int local[J], sum = 0;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int e = lane * J + j;
      local[j] = e < E ? cnt[e] : 0;
      sum += local[j];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int e = lane * J + j;
      if (e < E) {
        cursor[e] = run;
        offsets[e] = run;
      }
      run += local[j];
    }
    if (lane == 31) offsets[E] = incl;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int r0 = 0; r0 < n; r0 += blockDim.x) {
    const int i = r0 + tid;
    int e = -1;
    if (i < n && (m.counts == nullptr || (i % m.cap) < vc[i / m.cap])) {
      e = ids[i];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & lt_mask);
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    if (e >= 0) {
      int pos = cursor[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w][e];
      sorted_slots[pos] = i;
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < W; ++w) {
        add += wcnt[w][ee];
        wcnt[w][ee] = 0;
      }
      cursor[ee] += add;
    }
    __syncthreads();
  }
}

template <bool KPERM>
__global__ void permute_kernel(const uint4* __restrict__ x, int64_t n_rows, int vec_per_row, int k,
                               const int32_t* __restrict__ sorted_slots, uint4* __restrict__ xs,
                               const int32_t* __restrict__ n_dev) {
  // n_dev (optional): the number of sorted rows, known only on the device
  pdl_wait();
  const int64_t total = (n_dev != nullptr ? static_cast<int64_t>(*n_dev) : n_rows) * vec_per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = i / vec_per_row;
    const int v = static_cast<int>(i - p * vec_per_row);
    const int64_t tok = sorted_slots[p] / k;
    uint4 val = __ldg(x + tok * vec_per_row + v);
    if (KPERM) {
      const uint4 in = val;
      val.x = __byte_perm(in.x, in.z, 0x5410);
      val.y = __byte_perm(in.x, in.z, 0x7632);
      val.z = __byte_perm(in.y, in.w, 0x5410);
      val.w = __byte_perm(in.y, in.w, 0x7632);
    }
    xs[i] = val;
  }
}

__global__ void combine_kernel(const uint4* __restrict__ y, int64_t T, int k, int vec_per_row,
                               uint4* __restrict__ out) {
  pdl_wait();
  const int64_t total = T * vec_per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int v = static_cast<int>(i - t * vec_per_row);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const uint4 yv = __ldg(y + (t * k + j) * vec_per_row + v);
      const __nv_bfloat16* yp = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __bfloat162float(yp[q]));
    }
    uint4 o;
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = __float2bfloat16_rn(acc[q]);
    out[i] = o;
  }
}

// Expert-parallel dispatch: the rows of the (token, slot) entries in
// destination-rank order (sorted_slots from the alignment over ranks), each
// with its expert id local to the destination and its routed weight, plus the
// position at which each entry leaves (to put the returned rows back).
__global__ void ep_pack_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ topk_ids,
                               const float* __restrict__ topk_w, int64_t n, int vec_per_row, int k,
                               int experts_per_rank, const int32_t* __restrict__ sorted_slots,
                               uint4* __restrict__ rows, int32_t* __restrict__ local_ids,
                               float* __restrict__ weights, int32_t* __restrict__ inv_pos) {
  const int64_t total = n * vec_per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = i / vec_per_row;
    const int v = static_cast<int>(i - p * vec_per_row);
    const int32_t slot = sorted_slots[p];
    rows[i] = __ldg(x + static_cast<int64_t>(slot / k) * vec_per_row + v);
    if (v == 0) {
      const int32_t e = topk_ids[slot];
      local_ids[p] = e % experts_per_rank;
      weights[p] = topk_w[slot];
      inv_pos[slot] = static_cast<int32_t>(p);
    }
  }
}

// Expert-parallel combine: out[t] = bf16(sum_j back[inv_pos[t*k + j]]) in fp32, slot order.
__global__ void ep_combine_kernel(const uint4* __restrict__ back, const int32_t* __restrict__ inv_pos,
                                  int64_t T, int k, int vec_per_row, uint4* __restrict__ out) {
  const int64_t total = T * vec_per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int v = static_cast<int>(i - t * vec_per_row);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int64_t p = inv_pos[t * k + j];
      const uint4 yv = __ldg(back + p * vec_per_row + v);
      const __nv_bfloat16* yp = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __bfloat162float(yp[q]));
    }
    uint4 o;
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = __float2bfloat16_rn(acc[q]);
    out[i] = o;
  }
}

__global__ void ep_wait_kernel(const uint32_t* flags, int R, uint32_t epoch, uint64_t timeout_ns, int code) {
  if (threadIdx.x == 0) ep_wait_flags(flags, R, epoch, timeout_ns, code);
}

inline unsigned grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

}  // namespace

template <int TOK>
int launch_route(const void* x, const void* gate_w, int64_t T, int H, int E, int k, const float* bias,
                 int renormalize, void* logits, float* topk_w, int32_t* topk_ids, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(TOK) * H * 4 + static_cast<size_t>(TOK) * E * 4;
  if (smem > 200 * 1024) return fail(LLQ_EUNSUPPORTED, "hidden size %d too large for the router", H);
  static std::atomic<uint64_t> attr{0};
  if (first_use_on_device(attr))
    cudaFuncSetAttribute(route_kernel<TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  const unsigned blocks = static_cast<unsigned>((T + TOK - 1) / TOK);
  route_kernel<TOK><<<blocks, kRouteThreads, smem, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                         static_cast<const __nv_bfloat16*>(gate_w), T, H, E, k,
                                                         bias, renormalize, static_cast<__nv_bfloat16*>(logits),
                                                         topk_w, topk_ids);
  return check_launch("route_kernel");
}

int route_impl(const void* x, const void* gate_w, int64_t T, int H, int E, int k, const float* bias,
               int renormalize, void* logits, float* topk_w, int32_t* topk_ids, cudaStream_t st) {
  if (T <= 0) return LLQ_OK;
  if (E < 1 || E > kMaxExperts) return fail(LLQ_EUNSUPPORTED, "num_experts must be in [1, 256], got %d", E);
  if (k < 1 || k > E || k > 32) return fail(LLQ_EINVAL, "top_k must be in [1, min(E, 32)], got %d", k);
  if (H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8, got %d", H);
  // enough blocks to cover the SMs at decode sizes, more tokens per weight pass at prefill sizes
  if (E % 8 == 0 && E <= 64 && H % (kRmWarps * 32) == 0) {
    const size_t smem = static_cast<size_t>(kRmWarps) * 16 * E * 4;
    const unsigned blocks = static_cast<unsigned>((T + 15) / 16);
    auto* xp = static_cast<const __nv_bfloat16*>(x);
    auto* wp = static_cast<const __nv_bfloat16*>(gate_w);
    auto* lp = static_cast<__nv_bfloat16*>(logits);
#define LLQ_ROUTE_MMA(NT)                                                                                  \
  case NT: {                                                                                               \
    static std::atomic<uint64_t> attr{0};                                                                  \
    if (first_use_on_device(attr))                                                                         \
      cudaFuncSetAttribute(route_mma_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);  \
    launch_pdl(route_mma_kernel<NT>, dim3(blocks), dim3(kRmWarps * 32), smem, st, xp, wp, T, H, k, bias,    \
               renormalize, lp, topk_w, topk_ids);                                                         \
    return check_launch("route_mma_kernel");                                                               \
  }
    switch (E / 8) {
      LLQ_ROUTE_MMA(1)
      LLQ_ROUTE_MMA(2)
      LLQ_ROUTE_MMA(3)
      LLQ_ROUTE_MMA(4)
      LLQ_ROUTE_MMA(5)
      LLQ_ROUTE_MMA(6)
      LLQ_ROUTE_MMA(7)
      LLQ_ROUTE_MMA(8)
      default: break;
    }
#undef LLQ_ROUTE_MMA
  }
  const int sms = num_sms();
  int tok = T <= sms ? 1 : T <= 2 * sms ? 2 : T <= 8 * sms ? 4 : 8;
  if (static_cast<size_t>(tok) * H * 4 + static_cast<size_t>(tok) * E * 4 > 200 * 1024) tok = 1;
  switch (tok) {
    case 1: return launch_route<1>(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, st);
    case 2: return launch_route<2>(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, st);
    case 4: return launch_route<4>(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, st);
    default: return launch_route<8>(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, st);
  }
}

int route_topk_impl(const void* logits, int dtype, int64_t T, int E, int k, const float* bias,
                    int renormalize, float* topk_w, int32_t* topk_ids, cudaStream_t st) {
  if (T <= 0) return LLQ_OK;
  if (E < 1 || E > kMaxExperts) return fail(LLQ_EUNSUPPORTED, "num_experts must be in [1, 256], got %d", E);
  if (k < 1 || k > E || k > 32) return fail(LLQ_EINVAL, "top_k must be in [1, min(E, 32)], got %d", k);
  const unsigned blocks = static_cast<unsigned>((T * 32 + 255) / 256);
  if (dtype == LLQ_BF16)
    route_topk_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), T, E, k, bias, renormalize, topk_w, topk_ids);
  else if (dtype == LLQ_F32)
    route_topk_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(logits), T, E, k,
                                                     bias, renormalize, topk_w, topk_ids);
  else
    return fail(LLQ_EUNSUPPORTED, "logits dtype %d", dtype);
  return check_launch("route_topk_kernel");
}

size_t align_workspace_size(int64_t T, int k, int E) {
  const int64_t n = T * k;
  const int64_t nblk = (n + kAlignChunk - 1) / kAlignChunk;
  return static_cast<size_t>((nblk < 1 ? 1 : nblk) * E * sizeof(int32_t) + 256);
}

int align_impl_masked(const int32_t* ids, int64_t n, int E, int32_t* offsets, int32_t* sorted_slots, void* ws,
                      size_t ws_bytes, cudaStream_t st, const AlignMask& m) {
  if (E < 1 || E > kMaxExperts) return fail(LLQ_EUNSUPPORTED, "num_experts must be in [1, 256], got %d", E);
  if (m.counts != nullptr && (m.R < 1 || m.R > kMaxRanks || m.cap < 1))
    return fail(LLQ_EINVAL, "masked alignment needs 1 <= ranks <= %d and cap >= 1", kMaxRanks);
  if (ws_bytes < align_workspace_size(n, 1, E)) return fail(LLQ_ENOSPACE, "align workspace too small");
  if (n == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), st);
    return check_launch("align memset");
  }
  if (n <= kAlignSmallMax) {
    launch_pdl(align_small_kernel, dim3(1), dim3(kAlignSmallThreads), 0, st, ids, static_cast<int>(n), E, offsets,
               sorted_slots, m);
    return check_launch("align_small_kernel");
  }
  const int64_t nblk = (n + kAlignChunk - 1) / kAlignChunk;
  if (nblk > 0x7fffffff) return fail(LLQ_EINVAL, "too many entries");
  if (m.counts != nullptr && m.flags != nullptr) {
    ep_wait_kernel<<<1, 32, 0, st>>>(m.flags, m.R, m.epoch, m.timeout_ns, 0x502);
    int rc = check_launch("ep_wait_kernel");
    if (rc) return rc;
  }
  int32_t* counts = static_cast<int32_t*>(ws);
  align_count_kernel<<<static_cast<unsigned>(nblk), kAlignThreads, 0, st>>>(ids, n, E, counts, m);
  int rc = check_launch("align_count_kernel");
  if (rc) return rc;
  align_scan_kernel<<<1, kMaxExperts, 0, st>>>(counts, static_cast<int>(nblk), E, offsets);
  rc = check_launch("align_scan_kernel");
  if (rc) return rc;
  align_scatter_kernel<<<static_cast<unsigned>(nblk), kAlignThreads, 0, st>>>(ids, n, E, counts, sorted_slots, m);
  return check_launch("align_scatter_kernel");
}

int align_impl(const int32_t* ids, int64_t T, int k, int E, int32_t* offsets, int32_t* sorted_slots,
               void* ws, size_t ws_bytes, cudaStream_t st) {
  AlignMask m{};
  return align_impl_masked(ids, T * k, E, offsets, sorted_slots, ws, ws_bytes, st, m);
}

int permute_impl(const void* x, int64_t T, int H, int k, const int32_t* sorted_slots, void* xs,
                 cudaStream_t st, int kperm, const int32_t* n_dev) {
  if (H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8");
  const int64_t n = T * k;
  if (n == 0) return LLQ_OK;
  const int vpr = H / 8;
  if (kperm)
    launch_pdl(permute_kernel<true>, dim3(grid_for(n * vpr, 256)), dim3(256), 0, st, static_cast<const uint4*>(x), n,
               vpr, k, sorted_slots, static_cast<uint4*>(xs), n_dev);
  else
    launch_pdl(permute_kernel<false>, dim3(grid_for(n * vpr, 256)), dim3(256), 0, st, static_cast<const uint4*>(x),
               n, vpr, k, sorted_slots, static_cast<uint4*>(xs), n_dev);
  return check_launch("permute_kernel");
}

int ep_pack_impl(const void* x, const int32_t* topk_ids, const float* topk_w, int64_t T, int k, int H,
                 int experts_per_rank, const int32_t* sorted_slots, void* rows, int32_t* local_ids,
                 float* weights, int32_t* inv_pos, cudaStream_t st) {
  if (H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8");
  if (experts_per_rank < 1) return fail(LLQ_EINVAL, "experts_per_rank must be >= 1");
  const int64_t n = T * k;
  if (n == 0) return LLQ_OK;
  const int vpr = H / 8;
  ep_pack_kernel<<<grid_for(n * vpr, 256), 256, 0, st>>>(static_cast<const uint4*>(x), topk_ids, topk_w, n, vpr,
                                                         k, experts_per_rank, sorted_slots,
                                                         static_cast<uint4*>(rows), local_ids, weights, inv_pos);
  return check_launch("ep_pack_kernel");
}

int ep_combine_impl(const void* back, const int32_t* inv_pos, int64_t T, int k, int H, void* out, cudaStream_t st) {
  if (H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8");
  if (T == 0) return LLQ_OK;
  const int vpr = H / 8;
  ep_combine_kernel<<<grid_for(T * vpr, 256), 256, 0, st>>>(static_cast<const uint4*>(back), inv_pos, T, k, vpr,
                                                            static_cast<uint4*>(out));
  return check_launch("ep_combine_kernel");
}

int combine_impl(const void* y, int64_t T, int k, int H, void* out, cudaStream_t st) {
  if (H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8");
  if (T == 0) return LLQ_OK;
  const int vpr = H / 8;
  launch_pdl(combine_kernel, dim3(grid_for(T * vpr, 256)), dim3(256), 0, st, static_cast<const uint4*>(y), T, k, vpr,
             static_cast<uint4*>(out));
  return check_launch("combine_kernel");
}

}  // namespace llq
