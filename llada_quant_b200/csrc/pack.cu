// Quantize-and-pack, MSE scale search, dequantize and int4 (un)packing.
//
// Bit-exact restatement of src/LLaDA_Quant/algorithms/symmetric.py:
//   amax      = max |w| over the group (exact in the source dtype)      :117-119
//   s         = fp32(amax) / Qmax, IEEE division (not a reciprocal)      :119
//   MSE grid  = ratio_j = fp32(1 - max_shrink * j / grid) (double math),
//               cand = base * ratio_j, err = sum((round(w/safe) clamp * safe - w)^2)
//               with four separately rounded fp32 ops, strict '<' keeps the
//               earliest candidate                                       :188-204
//   q         = clamp(rint(w / safe), -Qmax-1, Qmax)                     :245-250
//   packing   = low nibble = even element, two's complement              :296-313
// Only the order of the per-group error sum differs from the reference's
// vectorised CPU reduction; the error terms themselves are identical.
//
// Layout: one warp per quantization group ("segment"); a row that the group
// size does not divide is a single segment (the per-row fallback of
// _as_groups, :85-90).  Each lane owns element pairs (2p, 2p+1), so an INT4
// lane writes whole bytes and the warp's stores are contiguous.
#include "llq_common.cuh"

namespace llq {

namespace {

constexpr int kPairsCached = 8;  // pairs per lane kept in registers (segments <= 512)

template <typename T>
__device__ __forceinline__ void load_pair(const T* seg, int64_t i, int seg_len, float& a, float& b) {
  a = (i < seg_len) ? to_f32<T>(seg[i]) : 0.f;
  b = (i + 1 < seg_len) ? to_f32<T>(seg[i + 1]) : 0.f;
}

__device__ __forceinline__ float quant_code(float x, float safe, float qmin, float qmax) {
  float t = rintf(__fdiv_rn(x, safe));
  return fminf(fmaxf(t, qmin), qmax);
}

// rint(x / safe) through the reciprocal: t = x * fl(1/safe) is within 3 ulps of the
// IEEE quotient fl(x / safe), so both round to the same integer unless a half-integer
// lies within that distance -- detected (|frac(t) - 1/2| < 2^-12, far wider than 3 ulps
// at the |t| <= 128.5 of INT4/INT8 codes) and then answered by the IEEE division itself.
__device__ __noinline__ float exact_code(float x, float safe) { return rintf(__fdiv_rn(x, safe)); }

__device__ __forceinline__ float quant_code_recip(float x, float safe, float inv, float qmin, float qmax) {
  const float t = __fmul_rn(x, inv);
  float r = rintf(t);
  // (also when t is huge, infinite or NaN: a subnormal scale whose reciprocal overflows)
  const bool near = fabsf(fabsf(t - r) - 0.5f) < 0x1p-12f || !(fabsf(t) <= 0x1p20f);
  if (__builtin_expect(near, 0)) r = exact_code(x, safe);
  return fminf(fmaxf(r, qmin), qmax);
}

// low byte of a code in [-128, 127] held as a float, without a float-to-int conversion:
// 1.5 * 2^23 + r keeps r, two's complement, in the low mantissa bits
__device__ __forceinline__ uint32_t code_bits(float r) { return __float_as_uint(__fadd_rn(r, 12582912.0f)); }

__device__ __forceinline__ float err_term(float x, float safe, float qmin, float qmax) {
  float t = quant_code(x, safe, qmin, qmax);
  float d = __fsub_rn(__fmul_rn(t, safe), x);
  return __fmul_rn(d, d);
}

__device__ __forceinline__ float apply_scale_round(float s, int scale_round) {
  if (scale_round == LLQ_BF16) return round_bf16(s);
  if (scale_round == LLQ_F16) return __half2float(__float2half_rn(s));
  return s;
}

// candidate ratio exactly as Python computes it, then the fp32 rounding that
// ATen applies to a double scalar multiplying a float32 tensor
__device__ __forceinline__ float grid_ratio(int step, int grid, double max_shrink) {
  double r = 1.0 - max_shrink * static_cast<double>(step) / static_cast<double>(grid);
  return static_cast<float>(r);
}

template <typename T, bool CACHED>
__global__ void __launch_bounds__(256) quantize_segments_kernel(
    const T* __restrict__ w, int64_t rows, int64_t K, int seg_len, int segs_per_row, int bits,
    int search, int grid, double max_shrink, int scale_round, int pack, int8_t* __restrict__ q,
    float* __restrict__ scale_out, float* __restrict__ errors_out) {
  const int lane = threadIdx.x & 31;
  const int64_t seg = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nseg = rows * segs_per_row;
  if (seg >= nseg) return;
  const int64_t row = seg / segs_per_row;
  const int g = static_cast<int>(seg % segs_per_row);
  const T* segp = w + row * K + static_cast<int64_t>(g) * seg_len;
  const int npairs = (seg_len + 1) >> 1;
  const float qmax = static_cast<float>((1 << (bits - 1)) - 1);
  const float qmin = -qmax - 1.f;

  float ca[kPairsCached], cb[kPairsCached];
  float amax = 0.f;
  if (CACHED) {
#pragma unroll
    for (int j = 0; j < kPairsCached; ++j) {
      const int p = lane + 32 * j;
      load_pair<T>(segp, 2 * static_cast<int64_t>(p), p < npairs ? seg_len : 0, ca[j], cb[j]);
      amax = fmaxf(amax, fmaxf(fabsf(ca[j]), fabsf(cb[j])));
    }
  } else {
    for (int p = lane; p < npairs; p += 32) {
      float a, b;
      load_pair<T>(segp, 2 * static_cast<int64_t>(p), seg_len, a, b);
      amax = fmaxf(amax, fmaxf(fabsf(a), fabsf(b)));
    }
  }
  amax = warp_max(amax);
  const float base = __fdiv_rn(amax, qmax);
  float chosen = base;

  if (search == LLQ_SEARCH_MSE) {
    float best = base;
    float best_err = __int_as_float(0x7f800000);  // +inf
    for (int step = 0; step < grid; ++step) {
      const float cand = __fmul_rn(base, grid_ratio(step, grid, max_shrink));
      const float safe = cand > 0.f ? cand : 1.f;
      float acc = 0.f;
      if (CACHED) {
#pragma unroll
        for (int j = 0; j < kPairsCached; ++j) {
          const int p = lane + 32 * j;
          if (p < npairs) {
            acc = __fadd_rn(acc, err_term(ca[j], safe, qmin, qmax));
            if (2 * p + 1 < seg_len) acc = __fadd_rn(acc, err_term(cb[j], safe, qmin, qmax));
          }
        }
      } else {
        for (int p = lane; p < npairs; p += 32) {
          float a, b;
          load_pair<T>(segp, 2 * static_cast<int64_t>(p), seg_len, a, b);
          acc = __fadd_rn(acc, err_term(a, safe, qmin, qmax));
          if (2 * p + 1 < seg_len) acc = __fadd_rn(acc, err_term(b, safe, qmin, qmax));
        }
      }
      const float err = warp_sum(acc);
      if (errors_out != nullptr && lane == 0) errors_out[seg * grid + step] = err;
      if (err < best_err) {
        best_err = err;
        best = cand;
      }
    }
    chosen = base > 0.f ? best : 0.f;
  }
  if (errors_out != nullptr) return;  // diagnostics call: no codes

  const float s = apply_scale_round(chosen, scale_round);
  const float safe = s > 0.f ? s : 1.f;
  if (lane == 0) scale_out[seg] = s;

  auto emit = [&](int p, float a, float b) {
    const int qa = static_cast<int>(quant_code(a, safe, qmin, qmax));
    const int qb = static_cast<int>(quant_code(b, safe, qmin, qmax));
    if (bits == 4 && pack) {
      // seg_len is even for packed INT4 (validated on the host)
      const int64_t byte = row * (K >> 1) + ((static_cast<int64_t>(g) * seg_len) >> 1) + p;
      q[byte] = static_cast<int8_t>((qa & 0xF) | ((qb & 0xF) << 4));
    } else {
      const int64_t e = row * K + static_cast<int64_t>(g) * seg_len + 2 * p;
      q[e] = static_cast<int8_t>(qa);
      if (2 * p + 1 < seg_len) q[e + 1] = static_cast<int8_t>(qb);
    }
  };
  if (CACHED) {
#pragma unroll
    for (int j = 0; j < kPairsCached; ++j) {
      const int p = lane + 32 * j;
      if (p < npairs) emit(p, ca[j], cb[j]);
    }
  } else {
    for (int p = lane; p < npairs; p += 32) {
      float a, b;
      load_pair<T>(segp, 2 * static_cast<int64_t>(p), seg_len, a, b);
      emit(p, a, b);
    }
  }
}

template <typename T>
int launch_quantize(const void* w, int64_t rows, int64_t K, int seg_len, int segs_per_row,
                    int bits, int search, int grid, double max_shrink, int scale_round, int pack,
                    int8_t* q, float* scale, float* errors, cudaStream_t st) {
  const int64_t nseg = rows * segs_per_row;
  const int threads = 256;
  const int64_t blocks = (nseg * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffff) return fail(LLQ_EINVAL, "quantize: too many groups (%lld)", (long long)nseg);
  const bool cached = ((seg_len + 1) / 2) <= 32 * kPairsCached;
  if (cached)
    quantize_segments_kernel<T, true><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
        static_cast<const T*>(w), rows, K, seg_len, segs_per_row, bits, search, grid, max_shrink,
        scale_round, pack, q, scale, errors);
  else
    quantize_segments_kernel<T, false><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
        static_cast<const T*>(w), rows, K, seg_len, segs_per_row, bits, search, grid, max_shrink,
        scale_round, pack, q, scale, errors);
  return check_launch("quantize_segments_kernel");
}

// ---------------------------------------------------------------------------
// bandwidth form of the amax path for the layout every checkpoint uses: bf16
// weights, 128-element groups that divide the row.  A group is 256 bytes, so a
// half-warp covers it with one 16-byte load per lane; the amax is a 4-step
// shuffle over the half-warp, and each lane writes its 8 codes as one 4-byte
// (packed INT4) or 8-byte (INT8) store -- the group's 64 or 128 output bytes
// leave as one contiguous half-warp store.  Same arithmetic as above: the exact
// bf16 amax, IEEE division by Qmax, rint of the IEEE quotient, clamp.
// ---------------------------------------------------------------------------
constexpr int kG128Unroll = 2;  // groups per half-warp per iteration (loads in flight)

template <bool PACK4>
__global__ void __launch_bounds__(256) quantize_g128_bf16_kernel(const uint4* __restrict__ w, int64_t ngroups,
                                                                 int bits, int scale_round,
                                                                 int8_t* __restrict__ q,
                                                                 float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 15;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const float qmax = static_cast<float>((1 << (bits - 1)) - 1);
  const float qmin = -qmax - 1.f;
  // each warp iteration covers 2 * kG128Unroll groups; the loop is warp-uniform so that
  // the half-warp shuffles always see a converged warp
  // software-pipelined: the next iteration's loads are in flight while this one computes
  const int64_t step = nwarps * 2 * kG128Unroll;
  uint4 nxt[kG128Unroll];
  auto load = [&](int64_t base, uint4 (&v)[kG128Unroll]) {
#pragma unroll
    for (int u = 0; u < kG128Unroll; ++u) {
      const int64_t g = base + 2 * u + (lane >> 4);
      v[u] = g < ngroups ? __ldcs(w + g * 16 + sub) : make_uint4(0, 0, 0, 0);
    }
  };
  load(warp * 2 * kG128Unroll, nxt);
  for (int64_t base = warp * 2 * kG128Unroll; base < ngroups; base += step) {
    uint4 v[kG128Unroll];
#pragma unroll
    for (int u = 0; u < kG128Unroll; ++u) v[u] = nxt[u];
    load(base + step, nxt);
#pragma unroll
    for (int u = 0; u < kG128Unroll; ++u) {
      const int64_t g = base + 2 * u + (lane >> 4);
      const uint32_t wd[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      float x[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(wd[i] << 16);
        x[2 * i + 1] = __uint_as_float(wd[i] & 0xFFFF0000u);
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = apply_scale_round(__fdiv_rn(amax, qmax), scale_round);
      const float safe = sc > 0.f ? sc : 1.f;
      const float inv = __frcp_rn(safe);
      if (g >= ngroups) continue;
      if (sub == 0) scale_out[g] = sc;
      uint32_t c[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = code_bits(quant_code_recip(x[i], safe, inv, qmin, qmax));
      if (PACK4) {
        uint32_t b = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) b |= (c[i] & 0xFu) << (4 * i);
        reinterpret_cast<uint32_t*>(q)[g * 16 + sub] = b;
      } else {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo |= (c[i] & 0xFFu) << (8 * i);
          hi |= (c[i + 4] & 0xFFu) << (8 * i);
        }
        reinterpret_cast<uint2*>(q)[g * 16 + sub] = make_uint2(lo, hi);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dequantize: 8 consecutive elements of one row per thread
// ---------------------------------------------------------------------------
template <typename OutT>
__device__ __forceinline__ OutT from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename OutT>
__global__ void dequantize_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                  int64_t rows, int64_t K, int bits, int group, int groups,
                                  int packed, OutT* __restrict__ out) {
  const int64_t total = rows * K;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 8;
  for (int64_t e0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; e0 < total;
       e0 += stride) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t e = e0 + i;
      if (e >= total) break;
      const int64_t row = e / K;
      const int64_t k = e - row * K;
      int v;
      if (bits == 4 && packed) {
        v = nibble(q[row * (K >> 1) + (k >> 1)], static_cast<int>(k & 1));
      } else {
        v = q[e];
      }
      const float s = scale[row * groups + (group > 0 ? k / group : 0)];
      out[e] = from_f32<OutT>(__fmul_rn(static_cast<float>(v), s));
    }
  }
}

// bf16 output, 16 elements (one scale) per thread: an 8-byte (INT4) or 16-byte
// (INT8) load, 32 bytes stored as two 16-byte stores; the row and scale index come
// from one 32-bit division per 16 elements.  Requires K % 16 == 0 and a group that
// is a multiple of 16 (or one scale per row).
template <bool INT4>
__global__ void __launch_bounds__(256) dequantize16_bf16_kernel(const int8_t* __restrict__ q,
                                                                const float* __restrict__ scale,
                                                                int64_t chunks, uint32_t chunks_per_row,
                                                                uint32_t chunks_per_group, int groups,
                                                                uint4* __restrict__ out) {
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < chunks;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = c / chunks_per_row;
    const uint32_t cr = static_cast<uint32_t>(c - row * chunks_per_row);
    const float s = __ldg(scale + row * groups + cr / chunks_per_group);
    int v[16];
    if (INT4) {
      const uint2 b = __ldcs(reinterpret_cast<const uint2*>(q) + c);
      const uint32_t w[2] = {b.x, b.y};
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = static_cast<int>(w[i >> 3] << (28 - 4 * (i & 7))) >> 28;
    } else {
      const uint4 b = __ldcs(reinterpret_cast<const uint4*>(q) + c);
      const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = static_cast<int>(w[i >> 2] << (24 - 8 * (i & 3))) >> 24;
    }
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __nv_bfloat162 p = __floats2bfloat162_rn(__fmul_rn(static_cast<float>(v[2 * i]), s),
                                               __fmul_rn(static_cast<float>(v[2 * i + 1]), s));
      o[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    __stcs(out + 2 * c, make_uint4(o[0], o[1], o[2], o[3]));
    __stcs(out + 2 * c + 1, make_uint4(o[4], o[5], o[6], o[7]));
  }
}

__global__ void pack_int4_kernel(const int8_t* __restrict__ v, int64_t npairs,
                                 int8_t* __restrict__ out, int32_t* __restrict__ range_error) {
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < npairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int a = v[2 * p], b = v[2 * p + 1];
    if (a < -8 || a > 7 || b < -8 || b > 7) atomicExch(range_error, 1);
    out[p] = static_cast<int8_t>((a & 0xF) | ((b & 0xF) << 4));
  }
}

__global__ void unpack_int4_kernel(const int8_t* __restrict__ packed, int64_t npairs,
                                   int8_t* __restrict__ out) {
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < npairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int8_t b = packed[p];
    out[2 * p] = static_cast<int8_t>(nibble(b, 0));
    out[2 * p + 1] = static_cast<int8_t>(nibble(b, 1));
  }
}

int segments(int64_t K, int group_size, int* seg_len, int* segs_per_row) {
  if (group_size == -1 || group_size <= 0 || K % group_size != 0) {
    if (K > 0x7fffffff) return fail(LLQ_EUNSUPPORTED, "row of %lld elements as one group", (long long)K);
    *seg_len = static_cast<int>(K);
    *segs_per_row = 1;
  } else {
    *seg_len = group_size;
    *segs_per_row = static_cast<int>(K / group_size);
  }
  return LLQ_OK;
}

}  // namespace

int quantize_impl(const void* w, int w_dtype, int64_t rows, int64_t K, int bits, int group_size,
                  int search, int grid, double max_shrink, int scale_round, int pack, int8_t* q,
                  float* scale, float* errors, cudaStream_t st) {
  if (bits != 4 && bits != 8) return fail(LLQ_EINVAL, "bits must be 8 or 4, got %d", bits);
  if (rows <= 0 || K <= 0) return fail(LLQ_EINVAL, "cannot quantize an empty tensor");
  if (w == nullptr || (errors == nullptr && (q == nullptr || scale == nullptr)))
    return fail(LLQ_EINVAL, "null pointer");
  if (search != LLQ_SEARCH_AMAX && search != LLQ_SEARCH_MSE)
    return fail(LLQ_EINVAL, "scale_search must be one of ['amax', 'mse']");
  if (search == LLQ_SEARCH_MSE && grid < 1) return fail(LLQ_EINVAL, "grid must be >= 1, got %d", grid);
  if (search == LLQ_SEARCH_MSE && !(max_shrink >= 0.0 && max_shrink < 1.0))
    return fail(LLQ_EINVAL, "max_shrink must lie in [0, 1), got %g", max_shrink);
  if (bits == 4 && pack) {
    if (K % 2 != 0)
      return fail(LLQ_EINVAL, "int4 packing needs an even last dimension, got K=%lld", (long long)K);
    if (group_size != -1 && group_size % 2 != 0)
      return fail(LLQ_EINVAL,
                  "int4 packing needs an even group_size so groups stay byte-aligned, got %d",
                  group_size);
  }
  int seg_len = 0, spr = 0;
  int rc = segments(K, group_size, &seg_len, &spr);
  if (rc) return rc;
  const bool aligned = (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 7) == 0;
  if (w_dtype == LLQ_BF16 && seg_len == 128 && search == LLQ_SEARCH_AMAX && errors == nullptr && aligned) {
    const int64_t ngroups = rows * spr;
    const int threads = 256;
    const int64_t need = (ngroups + 2 * kG128Unroll - 1) / (2 * kG128Unroll) * 32;
    const int64_t want = (need + threads - 1) / threads;
    const unsigned blocks = static_cast<unsigned>(want < num_sms() * 8 ? want : num_sms() * 8);
    if (bits == 4 && pack)
      quantize_g128_bf16_kernel<true><<<blocks, threads, 0, st>>>(static_cast<const uint4*>(w), ngroups, bits,
                                                                  scale_round, q, scale);
    else
      quantize_g128_bf16_kernel<false><<<blocks, threads, 0, st>>>(static_cast<const uint4*>(w), ngroups, bits,
                                                                   scale_round, q, scale);
    return check_launch("quantize_g128_bf16_kernel");
  }
  switch (w_dtype) {
    case LLQ_F32:
      return launch_quantize<float>(w, rows, K, seg_len, spr, bits, search, grid, max_shrink,
                                    scale_round, pack, q, scale, errors, st);
    case LLQ_F16:
      return launch_quantize<__half>(w, rows, K, seg_len, spr, bits, search, grid, max_shrink,
                                     scale_round, pack, q, scale, errors, st);
    case LLQ_BF16:
      return launch_quantize<__nv_bfloat16>(w, rows, K, seg_len, spr, bits, search, grid,
                                            max_shrink, scale_round, pack, q, scale, errors, st);
    default:
      return fail(LLQ_EUNSUPPORTED, "weight dtype %d", w_dtype);
  }
}

int dequantize_impl(const int8_t* q, const float* scale, int64_t rows, int64_t K, int bits,
                    int group_size, int packed, void* out, int out_dtype, cudaStream_t st) {
  if (bits != 4 && bits != 8) return fail(LLQ_EINVAL, "bits must be 8 or 4, got %d", bits);
  if (rows <= 0 || K <= 0) return LLQ_OK;
  if (packed && (bits != 4 || K % 2 != 0)) return fail(LLQ_EINVAL, "packed storage needs bits=4 and even K");
  const bool grouped = !(group_size == -1 || group_size <= 0 || K % group_size != 0);
  const int group = grouped ? group_size : 0;
  const int groups = grouped ? static_cast<int>(K / group_size) : 1;
  const bool vec_ok = out_dtype == LLQ_BF16 && K % 16 == 0 && (!grouped || group % 16 == 0) &&
                      (bits == 8 ? !packed : packed != 0) && K / 16 <= 0x7fffffff &&
                      (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec_ok) {
    const int64_t chunks = rows * K / 16;
    const uint32_t cpr = static_cast<uint32_t>(K / 16);
    const uint32_t cpg = grouped ? static_cast<uint32_t>(group / 16) : cpr;
    const int64_t want = (chunks + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(want < num_sms() * 8 ? want : num_sms() * 8);
    if (bits == 4)
      dequantize16_bf16_kernel<true><<<blocks, 256, 0, st>>>(q, scale, chunks, cpr, cpg, groups,
                                                             static_cast<uint4*>(out));
    else
      dequantize16_bf16_kernel<false><<<blocks, 256, 0, st>>>(q, scale, chunks, cpr, cpg, groups,
                                                              static_cast<uint4*>(out));
    return check_launch("dequantize16_bf16_kernel");
  }
  const int64_t work = (rows * K + 7) / 8;
  const int threads = 256;
  const int64_t want = (work + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(want < num_sms() * 16 ? want : num_sms() * 16);
  switch (out_dtype) {
    case LLQ_F32:
      dequantize_kernel<float><<<blocks, threads, 0, st>>>(q, scale, rows, K, bits, group, groups,
                                                           packed, static_cast<float*>(out));
      break;
    case LLQ_F16:
      dequantize_kernel<__half><<<blocks, threads, 0, st>>>(q, scale, rows, K, bits, group, groups,
                                                            packed, static_cast<__half*>(out));
      break;
    case LLQ_BF16:
      dequantize_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
          q, scale, rows, K, bits, group, groups, packed, static_cast<__nv_bfloat16*>(out));
      break;
    default:
      return fail(LLQ_EUNSUPPORTED, "output dtype %d", out_dtype);
  }
  return check_launch("dequantize_kernel");
}

int pack_int4_impl(const int8_t* v, int64_t n, int8_t* out, int32_t* range_error, cudaStream_t st) {
  if (n % 2 != 0) return fail(LLQ_EINVAL, "last dim must be even for int4 packing");
  if (n == 0) return LLQ_OK;
  const int64_t np = n / 2;
  const unsigned blocks = static_cast<unsigned>(np / 256 + 1 < 4096 ? np / 256 + 1 : 4096);
  pack_int4_kernel<<<blocks, 256, 0, st>>>(v, np, out, range_error);
  return check_launch("pack_int4_kernel");
}

int unpack_int4_impl(const int8_t* packed, int64_t n, int8_t* out, cudaStream_t st) {
  if (n % 2 != 0) return fail(LLQ_EINVAL, "int4 value count must be even");
  if (n == 0) return LLQ_OK;
  const int64_t np = n / 2;
  const unsigned blocks = static_cast<unsigned>(np / 256 + 1 < 4096 ? np / 256 + 1 : 4096);
  unpack_int4_kernel<<<blocks, 256, 0, st>>>(packed, np, out);
  return check_launch("unpack_int4_kernel");
}

}  // namespace llq
