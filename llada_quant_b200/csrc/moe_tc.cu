// tcgen05 grouped expert GEMMs over the packed LLaDA_Quant buffers (sm_100a).
//
// Shape of the work (swap-AB): the MMA's M side is 128 weight rows of one
// expert, its N side is that expert's routed tokens (16..128 per tile), K runs
// over the hidden (GEMM1) or intermediate (GEMM2) dimension in chunks of 128.
//
//   warp 0      TMA producer: packed weight tile(s) [128 rows x 64/128 bytes]
//               and the token tile [N rows x 128 bf16] into a 4-stage SMEM ring
//   warp 1      TMEM allocator and MMA issuer (one thread):
//               tcgen05.mma.cta_group::1.kind::f16, A from TMEM, B from SMEM
//   warps 2-9   dequantize: packed nibbles/bytes + fp32 group scale ->
//               bf16(q * s) exactly as dequantize_tensor
//               (src/LLaDA_Quant/algorithms/symmetric.py:286-293), written to
//               TMEM with tcgen05.st as the MMA's A operand; then the epilogue
//               (tcgen05.ld of the fp32 accumulators):
//                 GEMM1  h = bf16(bf16(silu(bf16(gate))) * bf16(up))
//                        (INFERENCE_REPO_CHANGES.md:296-309)
//                 GEMM2  y[slot] = bf16(acc * topk_w[slot])  (:259-265)
//
// The dequantized weights never touch HBM or SMEM: packed bytes stream
// HBM -> SMEM (TMA) -> registers -> TMEM.  No TMA multicast is used.
// Every mbarrier wait is bounded (about 2 s); on timeout the kernel records
// LLQ_ETIMEOUT-class codes in g_device_error, drains, frees TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "llq_common.cuh"

namespace llq {

namespace {

constexpr int KC = 128;        // K elements per pipeline step
constexpr int NT_MAX = 128;    // tokens per tile (MMA N <= 128)
constexpr int ROWS = 128;      // weight rows per MMA (M)
constexpr int DQ_WARPS = 8;    // two warpgroups of dequant/epilogue warps
constexpr int THREADS = 64 + DQ_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

template <bool GEMM1, int BITS>
struct Cfg {
  static constexpr int W_ROW_BYTES = KC * BITS / 8;             // 64 (int4) or 128 (int8)
  static constexpr int W_TILES = GEMM1 ? 2 : 1;                  // gate + up, or w2
  static constexpr int W_TILE_BYTES = ROWS * W_ROW_BYTES;
  static constexpr int W_STAGE_BYTES = W_TILES * W_TILE_BYTES;
  static constexpr int B_STAGE_BYTES = NT_MAX * KC * 2;
  static constexpr int STAGES = (GEMM1 && BITS == 8) ? 3 : 4;
  static constexpr int ACC_COLS = W_TILES * NT_MAX;
  static constexpr int A_STAGE_COLS = W_TILES * KC / 2;          // bf16 pairs per lane
  static constexpr int A_STAGES_FIT = (int)(TMEM_COLS - ACC_COLS) / A_STAGE_COLS;
  static constexpr int A_STAGES = A_STAGES_FIT > 4 ? 4 : A_STAGES_FIT;
  static constexpr int CHUNKS = KC * BITS / 8 / 16;              // 16-byte chunks per row per step
  static constexpr size_t SMEM_BYTES =
      1024 + static_cast<size_t>(STAGES) * (W_STAGE_BYTES + B_STAGE_BYTES) + 512;
};

struct TcArgs {
  const int32_t* offsets;
  const float* scale;
  const int32_t* sorted_slots;
  const float* topk_w;
  __nv_bfloat16* out;
  int K;           // reduction length (H for GEMM1, I for GEMM2)
  int rows_total;  // weight rows per expert (2I or H)
  int inter;       // I
  int n_out;       // output row length (I for GEMM1, H for GEMM2)
  int group;       // 0 = one scale per row
  int groups;      // scales per row
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(tx)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false if the CTA is aborting or the wait timed out (then it
// records `code` in the device error word and raises the CTA's abort flag).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                          int code) {
  if (mbar_try_wait(b, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(b, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicExch(&g_device_error, code);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = n
__device__ __forceinline__ uint32_t make_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(ROWS >> 4) << 24);
}

// shared-memory descriptor of a K-major, 128-byte-swizzled bf16 tile
// (rows of 128 bytes, 8-row atoms of 1024 bytes)
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// ---------------------------------------------------------------------------
// exact dequantization: bf16(fp32(q) * s), two values per bf16x2 word
// ---------------------------------------------------------------------------
// The integer is rebuilt as the float 2^23 + u (u = q + bias in the mantissa)
// and the bias subtracted exactly; the high nibble is taken in place, i.e.
// as 16 * q, and multiplied by s / 16 -- the same exact product, so the single
// fp32 rounding and the bf16 rounding match q * s in dequantize_tensor.
__device__ __forceinline__ uint32_t scale_pair_to_bf16x2(uint32_t lo_bits, uint32_t hi_bits, float c_lo,
                                                         float c_hi, float s_lo, float s_hi) {
  uint32_t o;
  asm("{\n\t.reg .b64 v, c, sc;\n\t"
      ".reg .f32 a, b;\n\t"
      "mov.b64 v, {%1, %2};\n\t"
      "mov.b64 c, {%3, %4};\n\t"
      "mov.b64 sc, {%5, %6};\n\t"
      "add.rn.f32x2 v, v, c;\n\t"
      "mul.rn.f32x2 v, v, sc;\n\t"
      "mov.b64 {a, b}, v;\n\t"
      "cvt.rn.bf16x2.f32 %0, b, a;\n\t}"
      : "=r"(o)
      : "r"(lo_bits), "r"(hi_bits), "f"(c_lo), "f"(c_hi), "f"(s_lo), "f"(s_hi));
  return o;
}

// 16 packed bytes = 32 int4 values -> 16 bf16x2 words (natural K order)
__device__ __forceinline__ void dequant_int4_chunk(uint4 v, float s, uint32_t (&out)[16]) {
  const float s16 = s * 0.0625f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = w[i] ^ 0x88888888u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t t = __byte_perm(x, 0x4B000000u, 0x7440u | j);
      out[i * 4 + j] = scale_pair_to_bf16x2(t & 0xFF00000Fu, t & 0xFF0000F0u, -8388616.f,
                                            -8388736.f, s, s16);
    }
  }
}

// 16 int8 values -> 8 bf16x2 words
__device__ __forceinline__ void dequant_int8_chunk(uint4 v, float s, uint32_t* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = w[i] ^ 0x80808080u;
    const uint32_t b0 = __byte_perm(x, 0x4B000000u, 0x7440u);
    const uint32_t b1 = __byte_perm(x, 0x4B000000u, 0x7441u);
    const uint32_t b2 = __byte_perm(x, 0x4B000000u, 0x7442u);
    const uint32_t b3 = __byte_perm(x, 0x4B000000u, 0x7443u);
    out[i * 2 + 0] = scale_pair_to_bf16x2(b0, b1, -8388736.f, -8388736.f, s, s);
    out[i * 2 + 1] = scale_pair_to_bf16x2(b2, b3, -8388736.f, -8388736.f, s, s);
  }
}

__device__ __forceinline__ int box_index(int rows) {
  return rows <= 16 ? 0 : rows <= 32 ? 1 : rows <= 64 ? 2 : 3;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <bool GEMM1, int BITS>
__global__ void __launch_bounds__(THREADS, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b0,
                       const __grid_constant__ CUtensorMap tm_b1, const __grid_constant__ CUtensorMap tm_b2,
                       const __grid_constant__ CUtensorMap tm_b3, const TcArgs args) {
  using C = Cfg<GEMM1, BITS>;
  constexpr int S = C::STAGES;
  constexpr int AS = C::A_STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sb = sw + S * C::W_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + S * C::B_STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* a_full = empty + S;
  uint64_t* a_empty = a_full + AS;
  uint64_t* acc_full = a_empty + AS;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.y, rb = blockIdx.x;
  const int row0 = args.offsets[e];
  const int m_e = args.offsets[e + 1] - row0;
  if (m_e <= 0) return;  // uniform for the whole CTA, before any barrier or TMEM use

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], DQ_WARPS + 1);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(&a_full[i], DQ_WARPS);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, DQ_WARPS);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_tiles = (m_e + NT_MAX - 1) / NT_MAX;
  const int kch = args.K / KC;
  const int total = n_tiles * kch;
  const int64_t wrow_a = static_cast<int64_t>(e) * args.rows_total + static_cast<int64_t>(rb) * ROWS;
  const int64_t wrow_b = wrow_a + args.inter;  // up rows (GEMM1 only)

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < total; ++it) {
        const int tile = it / kch, kc = it - tile * kch, s = it % S;
        if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, abort_flag, 0x100 + s)) break;
        const int rows_t = min(NT_MAX, m_e - tile * NT_MAX);
        const int bi = box_index(rows_t);
        const int box = 16 << bi;
        mbar_expect_tx(&full[s], C::W_STAGE_BYTES + 2 * box * 128);
        uint8_t* wdst = sw + s * C::W_STAGE_BYTES;
        tma_load_2d(wdst, &tm_w, kc * C::W_ROW_BYTES, static_cast<int>(wrow_a), &full[s]);
        if (GEMM1) tma_load_2d(wdst + C::W_TILE_BYTES, &tm_w, kc * C::W_ROW_BYTES, static_cast<int>(wrow_b), &full[s]);
        const CUtensorMap* tb = bi == 0 ? &tm_b0 : bi == 1 ? &tm_b1 : bi == 2 ? &tm_b2 : &tm_b3;
        uint8_t* bdst = sb + s * C::B_STAGE_BYTES;
        const int trow = row0 + tile * NT_MAX;
        tma_load_2d(bdst, tb, kc * KC, trow, &full[s]);
        tma_load_2d(bdst + box * 128, tb, kc * KC + 64, trow, &full[s]);
        ++issued;
      }
      // drain: never leave the CTA with copies still landing in its shared memory
      for (int it = (issued > S ? issued - S : 0); it < issued; ++it) {
        long long t0 = clock64();
        while (!mbar_try_wait(&full[it % S], (it / S) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t acc_a = tmem;                 // gate (GEMM1) or w2 accumulator
      const uint32_t acc_b = tmem + NT_MAX;        // up accumulator (GEMM1)
      const uint32_t a_base = tmem + C::ACC_COLS;
      for (int it = 0; it < total; ++it) {
        const int tile = it / kch, kc = it - tile * kch, s = it % S, sa = it % AS;
        if (kc == 0) {
          if (!mbar_wait(acc_empty, (tile & 1) ^ 1, abort_flag, 0x200)) break;
        }
        if (!mbar_wait(&full[s], (it / S) & 1, abort_flag, 0x210 + s)) break;
        if (!mbar_wait(&a_full[sa], (it / AS) & 1, abort_flag, 0x220 + sa)) break;
        tc_fence_after();
        const int rows_t = min(NT_MAX, m_e - tile * NT_MAX);
        const int nt = (rows_t + 15) & ~15;
        const int box = 16 << box_index(rows_t);
        const uint32_t idesc = make_idesc(nt);
        const uint32_t bbase = smem_u32(sb + s * C::B_STAGE_BYTES);
        const uint32_t a_stage = a_base + sa * C::A_STAGE_COLS;
#pragma unroll
        for (int j = 0; j < KC / 16; ++j) {
          const uint64_t bdesc = make_sdesc(bbase + (j >> 2) * box * 128 + (j & 3) * 32);
          const uint32_t acc = (kc > 0 || j > 0) ? 1u : 0u;
          tc_mma(acc_a, a_stage + j * 8, bdesc, idesc, acc);
          if (GEMM1) tc_mma(acc_b, a_stage + KC / 2 + j * 8, bdesc, idesc, acc);
        }
        tc_commit(&a_empty[sa]);
        tc_commit(&empty[s]);
        if (kc == kch - 1) tc_commit(acc_full);
      }
    }
  } else {
    // ------------------------------------------------------------- dequant + epilogue
    const int dw = warp - 2;            // 0..7
    const int wg = dw >> 2;             // warpgroup 0/1
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;        // weight row within the 128-row tile
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t a_base = tmem + C::ACC_COLS + lane_addr;
    // GEMM1: warpgroup 0 = gate rows, 1 = up rows (all chunks);
    // GEMM2: both on the same rows, warpgroup g takes half of the chunks.
    const int tile_sel = GEMM1 ? wg : 0;
    const int c_begin = GEMM1 ? 0 : wg * (C::CHUNKS / 2);
    const int c_end = GEMM1 ? C::CHUNKS : c_begin + C::CHUNKS / 2;
    const int64_t wrow = (tile_sel == 0 ? wrow_a : wrow_b) + r;
    const float* srow = args.scale + wrow * args.groups;
    bool ok = true;
    for (int it = 0; it < total && ok; ++it) {
      const int tile = it / kch, kc = it - tile * kch, s = it % S, sa = it % AS;
      if (!mbar_wait(&full[s], (it / S) & 1, abort_flag, 0x300 + s)) { ok = false; break; }
      if (!mbar_wait(&a_empty[sa], ((it / AS) & 1) ^ 1, abort_flag, 0x310 + sa)) { ok = false; break; }
      tc_fence_after();
      const float sc = srow[args.group > 0 ? (kc * KC) / args.group : 0];
      const uint8_t* wt = sw + s * C::W_STAGE_BYTES + tile_sel * C::W_TILE_BYTES + r * C::W_ROW_BYTES;
      const uint32_t a_stage = a_base + sa * C::A_STAGE_COLS + tile_sel * (KC / 2);
      if (BITS == 4) {
#pragma unroll
        for (int c = c_begin; c < c_end; ++c) {
          const int pc = c ^ ((r >> 1) & 3);  // 64-byte swizzle
          const uint4 v = *reinterpret_cast<const uint4*>(wt + pc * 16);
          uint32_t o[16];
          dequant_int4_chunk(v, sc, o);
          tc_st16(a_stage + c * 16, o);
        }
      } else {
#pragma unroll
        for (int c = c_begin; c < c_end; c += 2) {
          const uint4 v0 = *reinterpret_cast<const uint4*>(wt + ((c ^ (r & 7)) * 16));
          const uint4 v1 = *reinterpret_cast<const uint4*>(wt + (((c + 1) ^ (r & 7)) * 16));
          uint32_t o[16];
          dequant_int8_chunk(v0, sc, o);
          dequant_int8_chunk(v1, sc, o + 8);
          tc_st16(a_stage + c * 8, o);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[sa]);
        mbar_arrive(&empty[s]);
      }
      if (kc == kch - 1) {
        // ---- epilogue of this token tile
        if (!mbar_wait(acc_full, tile & 1, abort_flag, 0x320)) { ok = false; break; }
        tc_fence_after();
        const int rows_t = min(NT_MAX, m_e - tile * NT_MAX);
        const int nt = (rows_t + 15) & ~15;
        const int half = nt >> 1;
        const int n_glob = rb * ROWS + r;
        for (int t0 = wg * half; t0 < (wg + 1) * half; t0 += 8) {
          float va[8], vb[8];
          tc_ld8(tmem + lane_addr + t0, va);
          if (GEMM1) tc_ld8(tmem + lane_addr + NT_MAX + t0, vb);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int t = t0 + i;
            if (t >= rows_t) break;
            const int64_t p = static_cast<int64_t>(row0) + tile * NT_MAX + t;
            if (GEMM1) {
              const float g = round_bf16(va[i]);
              const float u = round_bf16(vb[i]);
              const float silu = round_bf16(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))));
              args.out[p * args.n_out + n_glob] = __float2bfloat16_rn(__fmul_rn(silu, u));
            } else {
              const int32_t slot = args.sorted_slots[p];
              args.out[static_cast<int64_t>(slot) * args.n_out + n_glob] =
                  __float2bfloat16_rn(__fmul_rn(va[i], args.topk_w[slot]));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LLQ_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_bytes & 15) != 0)
    return fail(LLQ_EINVAL, "TMA operands need 16-byte aligned bases and row strides");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LLQ_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return LLQ_OK;
}

template <bool GEMM1, int BITS>
int launch_tc(const void* act, int64_t n_rows, const int32_t* offsets, int E, int K, int rows_total,
              int inter, int n_out, const int8_t* q, const float* scale, int group_size,
              const int32_t* sorted_slots, const float* topk_w, void* out, cudaStream_t st) {
  using C = Cfg<GEMM1, BITS>;
  if (n_rows <= 0) return LLQ_OK;
  CUtensorMap tw, tb[4];
  const uint64_t k_bytes = static_cast<uint64_t>(K) * BITS / 8;
  int rc = make_map(&tw, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_bytes, static_cast<uint64_t>(E) * rows_total,
                    k_bytes, C::W_ROW_BYTES, ROWS,
                    BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  for (int i = 0; i < 4; ++i) {
    rc = make_map(&tb[i], act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, static_cast<uint64_t>(n_rows),
                  static_cast<uint64_t>(K) * 2, 64, 16u << i, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  TcArgs a;
  a.offsets = offsets;
  a.scale = scale;
  a.sorted_slots = sorted_slots;
  a.topk_w = topk_w;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.K = K;
  a.rows_total = rows_total;
  a.inter = inter;
  a.n_out = n_out;
  const bool grouped = group_size > 0 && K % group_size == 0;
  a.group = grouped ? group_size : 0;
  a.groups = grouped ? K / group_size : 1;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(moe_gemm_tc_kernel<GEMM1, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(C::SMEM_BYTES));
    attr = true;
  }
  dim3 grid(n_out / ROWS, E);
  moe_gemm_tc_kernel<GEMM1, BITS><<<grid, THREADS, C::SMEM_BYTES, st>>>(tw, tb[0], tb[1], tb[2], tb[3], a);
  return check_launch("moe_gemm_tc_kernel");
}

}  // namespace

bool tc_supported(int E, int N_out, int K, int bits, int group_size, bool gemm1) {
  (void)gemm1;
  if (bits != 4 && bits != 8) return false;
  if (E < 1 || E > 65535) return false;
  if (K % KC != 0 || N_out % ROWS != 0) return false;
  const bool grouped = group_size > 0 && K % group_size == 0;
  if (grouped && group_size % KC != 0) return false;  // one scale per 128-element step
  return true;
}

int gemm1_tc(const void* x_sorted, const int32_t* offsets, int64_t n_rows, int E, int H, int I,
             const int8_t* qw1, const float* sw1, int bits, int group_size, void* h_sorted,
             cudaStream_t st) {
  if (!tc_supported(E, I, H, bits, group_size, true))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM1: unsupported shape");
  if (bits == 4)
    return launch_tc<true, 4>(x_sorted, n_rows, offsets, E, H, 2 * I, I, I, qw1, sw1, group_size, nullptr,
                              nullptr, h_sorted, st);
  return launch_tc<true, 8>(x_sorted, n_rows, offsets, E, H, 2 * I, I, I, qw1, sw1, group_size, nullptr,
                            nullptr, h_sorted, st);
}

int gemm2_tc(const void* h_sorted, const int32_t* offsets, const int32_t* sorted_slots,
             const float* topk_w, int64_t n_rows, int E, int H, int I, const int8_t* qw2,
             const float* sw2, int bits, int group_size, void* y_slots, cudaStream_t st) {
  if (!tc_supported(E, H, I, bits, group_size, false))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM2: unsupported shape");
  if (bits == 4)
    return launch_tc<false, 4>(h_sorted, n_rows, offsets, E, I, H, 0, H, qw2, sw2, group_size,
                               sorted_slots, topk_w, y_slots, st);
  return launch_tc<false, 8>(h_sorted, n_rows, offsets, E, I, H, 0, H, qw2, sw2, group_size,
                             sorted_slots, topk_w, y_slots, st);
}

}  // namespace llq
