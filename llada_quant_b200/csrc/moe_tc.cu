// tcgen05 grouped expert GEMMs over the packed LLaDA_Quant buffers (sm_100a).
//
// Persistent kernel: one CTA per SM walks a compacted list of work items
// (expert, token tile, 256-row block).  Per item the MMA's M side is two
// 128-row weight tiles -- gate and up rows for GEMM1 (so the SiLU epilogue is
// thread-local), two consecutive 128-row blocks of w2 for GEMM2 -- and its N
// side is up to NTM of the expert's routed tokens.  K runs in steps of 128.
//
//   warp 0      TMA producer: per item the fp32 scales of both tiles (one bulk
//               copy each, double-buffered), per step both packed weight tiles
//               [128 rows x 64/128 B] and the token tile [N x 128] bf16
//   warp 1      TMEM allocator + MMA issuer (one thread):
//               tcgen05.mma.cta_group::1.kind::f16, A from TMEM, B from SMEM
//   warps 2-9   dequantize into TMEM (tcgen05.st) as the MMA's A operand
//   warps 10-17 epilogue (tcgen05.ld of the accumulators)
//
// Two dequantization modes:
//   exact  A = bf16(fp32(q) * s), bit-identical to dequantize_tensor
//          (src/LLaDA_Quant/algorithms/symmetric.py:286-293); one fp32
//          accumulator per tile over all of K.
//   fast   (INT4) A = q, the integer code, exact in bf16; the MMA writes one
//          fp32 partial sum per 128-group into a double-buffered TMEM slot and
//          the epilogue warps accumulate s_g * partial_g in fp32 registers --
//          the quantization contract W = q * s without rounding each weight to
//          bf16.  Codes are written in the order (k0,k4),(k1,k5),(k2,k6),(k3,k7)
//          of each 8-element block, so the token operand must be permuted the
//          same way (moe_permute with kperm, and GEMM1's epilogue for GEMM2).
// Epilogues follow the external fused_moe's rounding order:
//   GEMM1  h = bf16(bf16(silu(bf16(gate))) * bf16(up))  (INFERENCE_REPO_CHANGES.md:296-309)
//   GEMM2  y[slot] = bf16(acc * topk_w[slot])            (:259-265)
//
// No TMA multicast is used.  Every mbarrier wait is bounded (~2 s of SM
// clocks); on timeout the kernel records a code in g_device_error, drains its
// copies (bounded), frees TMEM and exits.
#include <cstdlib>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "llq_common.cuh"
#include "ep_window.cuh"

namespace llq {

namespace {

constexpr int KC = 128;
constexpr int ROWS = 128;
constexpr uint32_t TMEM_COLS = 512;
constexpr int MAX_G = 16;  // scale groups per row (K <= 2048 at group 128)
constexpr int MAX_E = 256;
constexpr long long kTimeoutCycles = 4000000000LL;

template <bool GEMM1, int BITS, bool FAST, int NTM>
struct Cfg {
  // BITS == 16: the weights are already bf16 (dequantized once per layer call for
  // prefill-sized batches) and reach the tensor cores from shared memory by TMA
  static constexpr bool SS = BITS == 16;
  // K per step: 128 (one scale group) for packed weights; 64 for bf16 weights, whose
  // stages are then small enough for 4-deep rings of both operands
  static constexpr int KS = SS ? 64 : KC;
  static constexpr int W_ROW_BYTES = KS * BITS / 8;  // packed bytes of one row per K step
  // a weight load brings 128 bytes of each row (two K steps at INT4): twice the
  // DRAM burst of one step, half the TMA row requests per weight byte
  static constexpr int W_STEPS = SS ? 1 : 128 / W_ROW_BYTES;
  static constexpr int W_LOAD_BYTES = W_ROW_BYTES * W_STEPS;
  static constexpr int W_TILE_BYTES = ROWS * W_LOAD_BYTES;
  static constexpr int W_STAGE_BYTES = 2 * W_TILE_BYTES;
  static constexpr int B_STAGE_BYTES = NTM * KS * 2;
  static constexpr int SCALE_BUF_BYTES = SS ? 0 : 2 * ROWS * MAX_G * 4;
  // Two rings: packed weights, released as soon as the dequantizing warps have
  // copied them to registers, and token tiles, released when the step's MMAs
  // complete.  Weight slots thus turn over at the speed of HBM, independently
  // of the MMA pipeline, and the weight ring takes what shared memory is left.
  static constexpr int B_STAGES = SS ? 4 : 3;
  static constexpr int W_STAGES_FIT =
      (220 * 1024 - 2 * SCALE_BUF_BYTES - B_STAGES * B_STAGE_BYTES) / W_STAGE_BYTES;
  static constexpr int W_STAGES = W_STAGES_FIT > 8 ? 8 : W_STAGES_FIT;
  // Warp roles.  A warp issues one tcgen05.mma per ~55 cycles whatever N is,
  // while a 128 x N x 16 MMA with N <= 64 runs in 16-32 cycles, so small-N
  // tiles are fed by several issuing warps: one per weight tile, optionally
  // one per (tile, even/odd 16-wide K slice) with its own accumulator (the
  // epilogue then adds the two halves).
  // (measured on B200 at C3: splitting K across four issuers with 16 dequant
  // warps gained nothing over two issuers with 8 -- exact dequantization is
  // then ALU-bound -- so SPLIT stays 1; the code keeps both layouts correct)
  static constexpr int SPLIT = 1;
  static constexpr int MMA_WARPS = 2 * SPLIT;
  // dequantizing warps: one warpgroup per weight tile (measured at C3: 16 warps, as
  // two per row or as two groups taking alternate K steps, gained nothing -- the
  // exact expansion is limited by its conversion and integer pipes, not latency)
  static constexpr int DQ_WARPS = SS ? 0 : 8;
  // token groups of one warpgroup each; the fast mode drains a partial sum every K step,
  // so it takes four warpgroups (measured: two-launch fast layer 176 -> 134 us), and so
  // does the bf16 prefill kernel, which has no dequantizing warps and whose epilogues
  // of 128-token tiles set its pace (measured: C4 step 95.2 -> 73.0 ms)
  static constexpr int EPI_WARPS = (FAST || SS) ? 16 : 8;
  static constexpr int FIRST_MMA = 2;  // warp 0 loads weights and scales, warp 1 token tiles
  static constexpr int FIRST_DQ = FIRST_MMA + MMA_WARPS;
  static constexpr int FIRST_EPI = FIRST_DQ + DQ_WARPS;
  static constexpr int THREADS = (FIRST_EPI + EPI_WARPS) * 32;
  // exact mode: the accumulators are double-buffered across items when they
  // fit beside two A stages, so that an item's epilogue overlaps the next
  // item's MMAs (64-token tiles); 128-token tiles keep one buffer
  static constexpr int ACC_BUFS = (!FAST && 2 * 2 * SPLIT * NTM <= (SS ? 512 : 256)) ? 2 : 1;
  static constexpr int ACC_BUF_COLS = 2 * SPLIT * NTM;
  static constexpr int ACC_COLS = FAST ? 4 * NTM : ACC_BUFS * ACC_BUF_COLS;
  static constexpr int A_STAGE_COLS = KC;  // 64 columns per tile
  static constexpr int A_STAGES_FIT = SS ? 2 : static_cast<int>(TMEM_COLS - ACC_COLS) / A_STAGE_COLS;
  static constexpr int A_STAGES = A_STAGES_FIT > 4 ? 4 : A_STAGES_FIT;
  static constexpr int CHUNKS = W_ROW_BYTES / 16;
  static constexpr size_t SMEM_BYTES =
      1024 + static_cast<size_t>(W_STAGES) * W_STAGE_BYTES + static_cast<size_t>(B_STAGES) * B_STAGE_BYTES +
      2 * SCALE_BUF_BYTES + 4096;
  static_assert(W_STAGES >= 2 && B_STAGES >= 2 && A_STAGES >= 2, "pipeline too shallow");
  static_assert(A_STAGES <= B_STAGES, "a TMEM A stage is released through the token ring");
  static_assert(!FAST || BITS == 4, "fast mode is INT4 only");
};

// one GEMM of the kernel (GEMM1 or GEMM2): its weights' scales, output and sizes
struct TcPhase {
  const float* scale;
  __nv_bfloat16* out;
  int K;           // reduction length (H for GEMM1, I for GEMM2)
  int rows_total;  // weight rows per expert (2I or H)
  int inter;       // I (GEMM1)
  int n_out;       // output row length (I for GEMM1, H for GEMM2)
  int rblocks;     // 256-row blocks per expert (I/128 for GEMM1, H/256 for GEMM2)
  int group;       // 0 = one scale per row
  int groups;      // scales per row
};

struct TcArgs {
  const int32_t* offsets;
  const int32_t* sorted_slots;
  const float* topk_w;
  TcPhase ph[2];   // ph[0] alone, or GEMM1 then GEMM2 when `fused`
  int fused;       // GEMM1 items, then GEMM2 items that wait for their token tile's GEMM1 items
  int* tile_done;  // fused: per token tile, GEMM1 epilogue warps finished; [tile_done_n] then a CTA counter
  int tile_done_n;
  int E;
  int dense_rows;  // offsets == nullptr: one expert of this many rows, identity slots, weight 1
  int ksplit;      // K slices per output tile (> 1: exact GEMM2 only, fp32 partials to `partial`)
  float* partial;  // [ksplit][rows][n_out] when ksplit > 1
  int ep_on;       // GEMM2 only: scatter rows into the peers' back regions and signal them
  EpScatter ep;
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

// try_wait that suspends the thread in hardware until the phase completes or
// `ns` nanoseconds pass, so that waiting warps take no issue slots from the
// dequantizing warps that share their SM sub-partition
__device__ __forceinline__ bool mbar_try_wait_for(uint64_t* b, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kSuspendNs = 200000;  // one suspended try_wait, 0.2 ms at most

// Bounded wait: false if the CTA is aborting or the wait timed out (then it
// records `code` in the device error word and raises the CTA's abort flag).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                          int code) {
  if (mbar_try_wait_for(b, parity, kSuspendNs)) return true;
  const long long t0 = clock64();
  while (true) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicExch(&g_device_error, code);
      return false;
    }
    if (mbar_try_wait_for(b, parity, kSuspendNs)) return true;
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

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 1 in exactly one lane of the (converged) warp, 0 in the others
__device__ __forceinline__ uint32_t elect_one() {
  uint32_t e;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(e));
  return e;
}

// issued by the lanes with `issue` != 0 (one per warp)
__device__ __forceinline__ void tc_mma(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate, uint32_t issue) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(issue)
      : "memory");
}

// A from shared memory (descriptor), for bf16 weights staged by TMA
__device__ __forceinline__ void tc_mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate, uint32_t issue) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(issue)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar, uint32_t issue) {
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(issue)
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

// 8 consecutive fp32 columns of this thread's TMEM lane; complete after tc_wait_ld()
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane; complete after tc_wait_ld()
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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
// dequantization
// ---------------------------------------------------------------------------
// exact: the integer is rebuilt as the float 2^23 + u (u = q + bias in the
// mantissa, byte permute) and the bias subtracted exactly; the high nibble is
// taken in place, i.e. as 16 * q, and multiplied by s / 16 -- the same exact
// product -- so the single fp32 rounding and the bf16 rounding equal those of
// q * s in dequantize_tensor.
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

// (x & mask) ^ k in one LOP3
__device__ __forceinline__ uint32_t and_xor(uint32_t x, uint32_t mask, uint32_t k) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(x), "r"(mask), "r"(k));
  return r;
}

// The four scale multipliers s * 2^-p (p = 0, 4, 8, 12) of one 128-group row.
struct NibbleScales {
  float s0, s4, s8, s12;
};

__device__ __forceinline__ NibbleScales nibble_scales(float s) {
  return NibbleScales{s, s * 0.0625f, s * 0.00390625f, s * 0.000244140625f};
}

// 16 packed bytes = 32 int4 values -> 16 bf16x2 words, natural K order.
// Each value is made a float by one LOP3 where it lies: nibble p of a word
// (p = 0, 4, 8, 12; the upper four nibbles after one shift by 16) becomes
// 2^23 + (q + 8) * 2^p, the bias 2^23 + 8 * 2^p is subtracted exactly and the
// product with s * 2^-p -- exactly q * s before its one fp32 rounding -- is
// rounded to bf16, as dequantize_tensor does.  Scales below 2^-100 (where
// s * 2^-12 would lose bits) take the byte-permute form, which only divides by 16.
__device__ __forceinline__ void dequant_int4_exact(uint4 v, float s, const NibbleScales& S, uint32_t (&out)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if (s >= 0x1p-100f) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t y = w[i] >> 16;
      out[i * 4 + 0] = scale_pair_to_bf16x2(and_xor(w[i], 0x0000000Fu, 0x4B000008u), and_xor(w[i], 0x000000F0u, 0x4B000080u),
                                            -8388616.f, -8388736.f, S.s0, S.s4);
      out[i * 4 + 1] = scale_pair_to_bf16x2(and_xor(w[i], 0x00000F00u, 0x4B000800u), and_xor(w[i], 0x0000F000u, 0x4B008000u),
                                            -8390656.f, -8421376.f, S.s8, S.s12);
      out[i * 4 + 2] = scale_pair_to_bf16x2(and_xor(y, 0x0000000Fu, 0x4B000008u), and_xor(y, 0x000000F0u, 0x4B000080u),
                                            -8388616.f, -8388736.f, S.s0, S.s4);
      out[i * 4 + 3] = scale_pair_to_bf16x2(and_xor(y, 0x00000F00u, 0x4B000800u), and_xor(y, 0x0000F000u, 0x4B008000u),
                                            -8390656.f, -8421376.f, S.s8, S.s12);
    }
    return;
  }
  const float s16 = s * 0.0625f;
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
__device__ __forceinline__ void dequant_int8_exact(uint4 v, float s, uint32_t* out) {
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

// fast: integer codes as bf16.  (x & 0x000F000F) ^ 0x43084308 puts nibbles 0
// and 4 into two bf16 mantissas as 128 + (q + 8); subtracting 136 leaves q
// exactly.  Pairs come out as (k0,k4),(k1,k5),(k2,k6),(k3,k7).
__device__ __forceinline__ uint32_t code_pair(uint32_t x) {
  uint32_t t, o;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43084308, 0x6A;" : "=r"(t) : "r"(x));
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(o) : "r"(t), "r"(0xC308C308u));
  return o;
}

__device__ __forceinline__ void codes_int4(uint4 v, uint32_t (&out)[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[i * 4 + 0] = code_pair(w[i]);
    out[i * 4 + 1] = code_pair(w[i] >> 4);
    out[i * 4 + 2] = code_pair(w[i] >> 8);
    out[i * 4 + 3] = code_pair(w[i] >> 12);
  }
}

// position of feature n inside a K-permuted row (inverse of [0,4,1,5,2,6,3,7])
__device__ __forceinline__ int kperm_pos(int n) {
  const int j = n & 7;
  return (n & ~7) | (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

// SiLU's quotient g / d (d = 1 + exp(-g) >= 1) as the bf16 value of its correctly
// rounded fp32 form, without the IEEE division in the common case: the quotient
// from the approximate reciprocal lies within 2 ulp of g / d, so it rounds to the
// same bf16 value unless it lies within 8 ulp of a bf16 rounding midpoint (low 16
// bits 0x8000); those, and d beyond 2^120 or not finite, are flagged in `need`
// for __fdiv_rn.
__device__ __forceinline__ float silu_quot_fast(float g, float d, bool& need) {
  const float q = __fdividef(g, d);
  const uint32_t lo = __float_as_uint(q) & 0xFFFFu;
  need = (lo - 0x7FF8u) <= 16u || !(d < 0x1p120f);
  return q;
}

__device__ __forceinline__ int box_index(int rows) {
  return rows <= 16 ? 0 : rows <= 32 ? 1 : rows <= 64 ? 2 : 3;
}

struct Item {
  int e, tt, tg, rb, row0, rows_t, ks, ph;
};

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <bool GEMM1, int BITS, bool FAST, int NTM>
__global__ void __launch_bounds__((Cfg<GEMM1, BITS, FAST, NTM>::THREADS), 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_b00,
                       const __grid_constant__ CUtensorMap tm_b01, const __grid_constant__ CUtensorMap tm_b02,
                       const __grid_constant__ CUtensorMap tm_b03, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_b10, const __grid_constant__ CUtensorMap tm_b11,
                       const __grid_constant__ CUtensorMap tm_b12, const __grid_constant__ CUtensorMap tm_b13,
                       const TcArgs args) {
  using C = Cfg<GEMM1, BITS, FAST, NTM>;
  constexpr int WS = C::W_STAGES;
  constexpr int BS = C::B_STAGES;
  constexpr int AS = C::A_STAGES;
  constexpr int SPLIT = C::SPLIT;
  constexpr int MMA_WARPS = C::MMA_WARPS;
  constexpr int DQ_WARPS = C::DQ_WARPS;
  constexpr int FIRST_MMA = C::FIRST_MMA;
  constexpr int FIRST_DQ = C::FIRST_DQ;
  constexpr int FIRST_EPI = C::FIRST_EPI;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sw = smem;
  uint8_t* sb = sw + WS * C::W_STAGE_BYTES;
  float* ssc = reinterpret_cast<float*>(sb + BS * C::B_STAGE_BYTES);  // [2 bufs][2 tiles][128 * G]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(ssc) + 2 * C::SCALE_BUF_BYTES);
  uint64_t* wfull = bars;               // [WS] weight tiles landed
  uint64_t* wfree = wfull + WS;         // [WS] dequant warps have read the weight tiles
  uint64_t* bfull = wfree + WS;         // [BS] token tile landed
  uint64_t* mdone = bfull + BS;         // [BS] the step's MMAs completed (one commit per step)
  uint64_t* a_full = mdone + BS;        // [2 tiles][AS]: TMEM A stage written
  uint64_t* sc_full = a_full + 2 * AS;  // [2]
  uint64_t* sc_empty = sc_full + 2;     // [2]
  uint64_t* acc_full = sc_empty + 2;    // [2] (per item in exact mode, per step in fast mode)
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* tile_prefix = reinterpret_cast<int*>(tmem_slot + 2);  // [E + 1]
  int* row_offsets = tile_prefix + MAX_E + 1;                // [E + 1]: the expert offsets, staged once

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.E;
  pdl_wait();
  // the previous kernel's generic stores (the token rows this launch reads) must be
  // visible to this launch's TMA (async proxy) reads
  asm volatile("fence.proxy.async.global;" ::: "memory");
  // phase of an item: 0 = GEMM1 (or the single GEMM), 1 = GEMM2 of a fused launch
  auto is_g1 = [&](int ph) -> bool { return args.fused ? ph == 0 : GEMM1; };

  // ---- compacted work list: token tiles per expert, prefix-summed by warp 0
  if (warp == 0) {
    int local[MAX_E / 32];
    int sum = 0;
#pragma unroll
    for (int j = 0; j < MAX_E / 32; ++j) {
      const int e = lane * (MAX_E / 32) + j;
      int n = 0;
      if (e < E) {
        const int o0 = args.offsets != nullptr ? args.offsets[e] : 0;
        const int m = args.offsets != nullptr ? args.offsets[e + 1] - o0 : args.dense_rows;
        row_offsets[e] = o0;
        if (e == E - 1) row_offsets[E] = o0 + m;
        n = (m + NTM - 1) / NTM;
      }
      local[j] = n;
      sum += n;
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
#pragma unroll
    for (int j = 0; j < MAX_E / 32; ++j) {
      const int e = lane * (MAX_E / 32) + j;
      if (e < E) tile_prefix[e] = run;
      run += local[j];
    }
    if (lane == 31) tile_prefix[E] = incl;
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < WS; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wfree[i], C::SS ? MMA_WARPS : DQ_WARPS);
    }
    for (int i = 0; i < BS; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&mdone[i], MMA_WARPS);
    }
    for (int i = 0; i < 2 * AS; ++i) mbar_init(&a_full[i], 4);  // the tile's warpgroup of the step's group
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], C::SS ? 1 : (FAST ? DQ_WARPS + C::EPI_WARPS : DQ_WARPS));
      mbar_init(&acc_full[i], MMA_WARPS);
      mbar_init(&acc_empty[i], C::EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == FIRST_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total_tiles = tile_prefix[E];
  const int items0 = total_tiles * args.ph[0].rblocks * args.ksplit;
  const int total_items = items0 + (args.fused ? total_tiles * args.ph[1].rblocks : 0);

  auto item_at = [&](int u) -> Item {
    Item it;
    it.ph = u >= items0 ? 1 : 0;
    const int ks = it.ph ? 1 : args.ksplit;
    const int v = it.ph ? u - items0 : u;
    const int uu = v / ks;
    it.ks = v - uu * ks;
    const int rbl = args.ph[it.ph].rblocks;
    const int tg = uu / rbl;
    it.tg = tg;
    it.rb = uu - tg * rbl;
    int lo = 0, hi = E;  // largest e with tile_prefix[e] <= tg
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (tile_prefix[mid] <= tg) lo = mid; else hi = mid;
    }
    it.e = lo;
    it.tt = tg - tile_prefix[lo];
    const int base = row_offsets[lo];
    const int m = row_offsets[lo + 1] - base;
    it.row0 = base + it.tt * NTM;
    it.rows_t = min(NTM, m - it.tt * NTM);
    return it;
  };
  auto wrow_of = [&](const Item& it, int tile) -> int64_t {
    const TcPhase& P = args.ph[it.ph];
    if (is_g1(it.ph))
      return static_cast<int64_t>(it.e) * P.rows_total + (tile ? P.inter : 0) + static_cast<int64_t>(it.rb) * ROWS;
    return static_cast<int64_t>(it.e) * P.rows_total + static_cast<int64_t>(it.rb) * 2 * ROWS + tile * ROWS;
  };
  // K steps of an item: [kbeg, kbeg + kper)
  auto k_range = [&](const Item& it, int& kbeg, int& kper) {
    const int kch = args.ph[it.ph].K / C::KS;
    kper = kch / (it.ph ? 1 : args.ksplit);
    kbeg = it.ks * kper;
  };

  if (warp == 0) {
    // ------------------------------------------------------- weight producer
    // per item the fp32 scales of both tiles, per K step both packed weight tiles
    if (lane == 0) {
      int issued = 0, rs = 0;
      uint32_t rph = 0;  // weight ring slot and phase
      bool ok = true;
      for (int u = blockIdx.x, ii = 0; u < total_items && ok; u += gridDim.x, ++ii) {
        const Item item = item_at(u);
        const TcPhase& P = args.ph[item.ph];
        const int G = P.groups;
        const int sbuf = ii & 1;
        if (!C::SS) {
          if (!mbar_wait(&sc_empty[sbuf], ((ii >> 1) & 1) ^ 1, abort_flag, 0x100)) break;
          const uint32_t sbytes = static_cast<uint32_t>(ROWS * G * 4);
          mbar_expect_tx(&sc_full[sbuf], 2 * sbytes);
          float* sdst = ssc + sbuf * (2 * ROWS * MAX_G);
          bulk_load(sdst, P.scale + wrow_of(item, 0) * G, sbytes, &sc_full[sbuf]);
          bulk_load(sdst + ROWS * MAX_G, P.scale + wrow_of(item, 1) * G, sbytes, &sc_full[sbuf]);
        }
        const CUtensorMap* tw = item.ph == 0 ? &tm_w0 : &tm_w1;
        const int w0 = static_cast<int>(wrow_of(item, 0)), w1 = static_cast<int>(wrow_of(item, 1));
        int kbeg, kper;
        k_range(item, kbeg, kper);
        for (int kc = kbeg; kc < kbeg + kper; kc += C::W_STEPS) {
          if (!mbar_wait(&wfree[rs], rph ^ 1, abort_flag, 0x110 + rs)) { ok = false; break; }
          mbar_expect_tx(&wfull[rs], C::W_STAGE_BYTES);
          uint8_t* wdst = sw + rs * C::W_STAGE_BYTES;
          if (C::SS) {  // bf16 rows: two 64-element, 128-byte-swizzled boxes per tile
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              tma_load_2d(wdst + t * C::W_TILE_BYTES, tw, kc * C::KS, t ? w1 : w0, &wfull[rs]);
            }
          } else {
            tma_load_2d(wdst, tw, kc * C::W_ROW_BYTES, w0, &wfull[rs]);
            tma_load_2d(wdst + C::W_TILE_BYTES, tw, kc * C::W_ROW_BYTES, w1, &wfull[rs]);
          }
          ++issued;
          if (++rs == WS) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
      // never leave copies in flight into this CTA's shared memory
      for (int i = (issued > WS ? issued - WS : 0); i < issued; ++i) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&wfull[i % WS], (i / WS) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- token producer
    // per K step the token tile [rows x 128] bf16, into a slot the step's MMAs released
    if (lane == 0) {
      int issued = 0, rs = 0;
      uint32_t rph = 0;  // token ring slot and phase
      bool ok = true;
      for (int u = blockIdx.x; u < total_items && ok; u += gridDim.x) {
        const Item item = item_at(u);
        if (item.ph == 1) {
          // the GEMM1 items of this token tile (every epilogue warp of each) must have stored h
          const int need = args.ph[0].rblocks * C::EPI_WARPS;
          const long long t0 = clock64();
          bool ready = false;
          while (!(ready = ld_acquire_gpu(args.tile_done + item.tg) >= need)) {
            if (*abort_flag) break;
            if (clock64() - t0 > kTimeoutCycles) {
              *abort_flag = 1;
              atomicExch(&g_device_error, 0x130);
              break;
            }
            __nanosleep(64);
          }
          if (!ready) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");  // generic stores of h -> TMA reads
        }
        const int bi = box_index(item.rows_t);
        const int box = 16 << bi;
        const CUtensorMap* tb =
            item.ph == 0 ? (bi == 0 ? &tm_b00 : bi == 1 ? &tm_b01 : bi == 2 ? &tm_b02 : &tm_b03)
                         : (bi == 0 ? &tm_b10 : bi == 1 ? &tm_b11 : bi == 2 ? &tm_b12 : &tm_b13);
        int kbeg, kper;
        k_range(item, kbeg, kper);
        for (int kc = kbeg; kc < kbeg + kper; ++kc) {
          if (!mbar_wait(&mdone[rs], rph ^ 1, abort_flag, 0x118 + rs)) { ok = false; break; }
          mbar_expect_tx(&bfull[rs], (C::KS / 64) * box * 128);
          uint8_t* bdst = sb + rs * C::B_STAGE_BYTES;
          tma_load_2d(bdst, tb, kc * C::KS, item.row0, &bfull[rs]);
          if (C::KS == 128) tma_load_2d(bdst + box * 128, tb, kc * C::KS + 64, item.row0, &bfull[rs]);
          ++issued;
          if (++rs == BS) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
      for (int i = (issued > BS ? issued - BS : 0); i < issued; ++i) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&bfull[i % BS], (i / BS) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else if (warp < FIRST_DQ) {
    // ------------------------------------------------------------- MMA issuers
    const int tile = (warp - FIRST_MMA) & 1;   // weight tile
    const int par = (warp - FIRST_MMA) >> 1;   // K-slice parity (SPLIT == 2)
    // the whole warp runs the loop (its descriptor arithmetic stays warp-uniform);
    // one elected lane issues the MMAs and the commits that track them
    const uint32_t leader = elect_one();
    {
      const uint32_t a_base = tmem + C::ACC_COLS;
      int it = 0, rs = 0, ra = 0, ws = 0;
      uint32_t rph = 0, raph = 0, wph = 0;  // token ring, TMEM A stage, (SS) weight ring: slots and phases
      bool ok = true;
      for (int u = blockIdx.x, ii = 0; u < total_items && ok; u += gridDim.x, ++ii) {
        const Item item = item_at(u);
        const int nt = (item.rows_t + 15) & ~15;
        const int box = 16 << box_index(item.rows_t);
        const uint32_t idesc = make_idesc(nt);
        if (!FAST) {
          const int ab = C::ACC_BUFS == 2 ? (ii & 1) : 0;
          const uint32_t ph = C::ACC_BUFS == 2 ? ((ii >> 1) & 1) : (ii & 1);
          if (!mbar_wait(&acc_empty[ab], ph ^ 1, abort_flag, 0x200)) break;
          tc_fence_after();
        }
        int kbeg, kper;
        k_range(item, kbeg, kper);
        const int kend = kbeg + kper;
        for (int kc = kbeg; kc < kend; ++kc, ++it) {
          const int s = rs, sa = ra;
          const uint32_t acc_base = tmem + (C::ACC_BUFS == 2 ? (ii & 1) * C::ACC_BUF_COLS : 0);
          uint32_t d0 = acc_base + par * NTM, d1 = acc_base + (SPLIT + par) * NTM;
          if (FAST) {
            const int pb = it & 1;
            if (!mbar_wait(&acc_empty[pb], ((it >> 1) & 1) ^ 1, abort_flag, 0x210 + pb)) { ok = false; break; }
            d0 = tmem + pb * 2 * NTM;
            d1 = d0 + NTM;
          }
          if (!mbar_wait(&bfull[s], rph, abort_flag, 0x220 + s)) { ok = false; break; }
          if (C::SS) {
            if (!mbar_wait(&wfull[ws], wph, abort_flag, 0x240 + ws)) { ok = false; break; }
          } else if (!mbar_wait(&a_full[tile * AS + sa], raph, abort_flag, 0x230 + sa)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors advance by plain adds on the 16-byte-unit start address
          const uint64_t bdesc0 = make_sdesc(smem_u32(sb + s * C::B_STAGE_BYTES));
          const uint64_t half_step = static_cast<uint64_t>((box * 128) >> 4);
          const uint32_t a_stage = a_base + sa * C::A_STAGE_COLS + tile * (KC / 2);
          const uint32_t d = tile ? d1 : d0;
          const uint32_t first = FAST ? 0u : (kc > kbeg ? 1u : 0u);
#pragma unroll
          for (int jj = 0; jj < C::KS / 16 / SPLIT; ++jj) {
            const int j = jj * SPLIT + par;
            const uint64_t bdesc = bdesc0 + (j >> 2) * half_step + (j & 3) * 2;
            const uint32_t acc = jj > 0 ? 1u : first;
            if (C::SS) {
              // A = this tile's bf16 weights in shared memory, laid out like the token tile
              const uint64_t adesc = make_sdesc(smem_u32(sw + ws * C::W_STAGE_BYTES + tile * C::W_TILE_BYTES)) +
                                     (j >> 2) * static_cast<uint64_t>((ROWS * 128) >> 4) + (j & 3) * 2;
              tc_mma_ss(d, adesc, bdesc, idesc, acc, leader);
            } else {
              tc_mma(d, a_stage + j * 8, bdesc, idesc, acc, leader);
            }
          }
          tc_commit(&mdone[s], leader);
          if (C::SS) {  // the step's MMAs also release the weight stage
            tc_commit(&wfree[ws], leader);
            if (++ws == WS) {
              ws = 0;
              wph ^= 1;
            }
          }
          if (!FAST && kc == kend - 1) tc_commit(&acc_full[C::ACC_BUFS == 2 ? (ii & 1) : 0], leader);
          if (++rs == BS) {
            rs = 0;
            rph ^= 1;
          }
          if (++ra == AS) {
            ra = 0;
            raph ^= 1;
          }
        }
      }
    }
  } else if (warp < FIRST_EPI) {
    // ------------------------------------------------------------- dequant
    const int wg = ((warp - FIRST_DQ) >> 2) & 1;  // weight tile
    const int q = warp & 3;                 // TMEM lane quarter
    const int r = q * 32 + lane;            // row within the tile
    const uint32_t a_row = tmem + C::ACC_COLS + (static_cast<uint32_t>(q * 32) << 16) + wg * (KC / 2);
    // weight ring slot of step it, token ring slot of step it - AS (whose MMAs
    // release TMEM A stage it % AS), TMEM A stage of step it, and their phases
    int it = 0, rs = 0, ps = BS - AS, ra = 0;
    uint32_t rph = 0, pph = 1;
    bool ok = true;
    for (int u = blockIdx.x, ii = 0; u < total_items && ok; u += gridDim.x, ++ii) {
      const Item item = item_at(u);
      const TcPhase& P = args.ph[item.ph];
      const int sbuf = ii & 1;
      if (!mbar_wait(&sc_full[sbuf], (ii >> 1) & 1, abort_flag, 0x300)) break;
      const float* srow = ssc + sbuf * (2 * ROWS * MAX_G) + wg * (ROWS * MAX_G) + r * P.groups;
      const int spg = P.group / KC;  // K steps per scale group (0: one scale per row)
      int kbeg, kper;
      k_range(item, kbeg, kper);
      for (int kc = kbeg; kc < kbeg + kper; ++kc, ++it) {
        const int s = rs, sa = ra;
        const int half = (kc - kbeg) % C::W_STEPS;  // K step within the weight stage
        const bool stage_done = half == C::W_STEPS - 1 || kc == kbeg + kper - 1;
        const float sc = FAST ? 0.f : srow[spg == 1 ? kc : spg == 0 ? 0 : kc / spg];
        const NibbleScales nsc = nibble_scales(sc);
        if (!mbar_wait(&wfull[s], rph, abort_flag, 0x310 + s)) { ok = false; break; }
        const uint8_t* wt = sw + s * C::W_STAGE_BYTES + wg * C::W_TILE_BYTES + r * C::W_LOAD_BYTES;
        const uint32_t a_stage = a_row + sa * C::A_STAGE_COLS;
        // this row's packed bytes into registers, then hand the weight slot back
        // to the producer at once; only the token tile waits for the MMA
        constexpr int MYC = C::CHUNKS;
        uint4 v[MYC];
#pragma unroll
        for (int ci = 0; ci < MYC; ++ci) {
          const int c = half * C::CHUNKS + ci;
          const int pc = c ^ (r & 7);  // 128-byte swizzle
          v[ci] = *reinterpret_cast<const uint4*>(wt + pc * 16);
        }
        // our generic reads of the stage before the TMA (async proxy) refills it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (stage_done && lane == 0) mbar_arrive(&wfree[s]);
        // the TMEM A stage is free once the MMAs of step it - AS completed
        if (it >= AS && !mbar_wait(&mdone[ps], pph, abort_flag, 0x320 + sa)) { ok = false; break; }
        tc_fence_after();
        if (BITS == 4) {
#pragma unroll
          for (int ci = 0; ci < MYC; ++ci) {
            uint32_t o[16];
            if (FAST) codes_int4(v[ci], o);
            else dequant_int4_exact(v[ci], sc, nsc, o);
            tc_st16(a_stage + ci * 16, o);
          }
        } else {
#pragma unroll
          for (int ci = 0; ci < MYC; ci += 2) {
            uint32_t o[16];
            dequant_int8_exact(v[ci], sc, o);
            dequant_int8_exact(v[ci + 1], sc, o + 8);
            tc_st16(a_stage + ci * 8, o);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[wg * AS + sa]);
        if (stage_done && ++rs == WS) {
          rs = 0;
          rph ^= 1;
        }
        if (++ps == BS) {
          ps = 0;
          pph ^= 1;
        }
        if (++ra == AS) ra = 0;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // scale reads before the bulk refill
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&sc_empty[sbuf]);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int eg = (warp - FIRST_EPI) >> 2;  // token half
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    constexpr int EG = C::EPI_WARPS / 4;  // token groups, one epilogue warpgroup each
    constexpr int HALF = NTM / EG;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x, ii = 0; u < total_items && ok; u += gridDim.x, ++ii) {
      const Item item = item_at(u);
      const TcPhase& P = args.ph[item.ph];
      const bool g1 = is_g1(item.ph);
      const int nt = (item.rows_t + 15) & ~15;
      const int t_begin = eg * (nt / EG), t_end = (eg + 1) * (nt / EG);
      // GEMM2: the (token, slot) destination and routed weight of this warp's tokens,
      // one token per lane, loaded before the accumulators are ready and broadcast
      // by shuffles below (a dependent pair of global loads per token otherwise)
      constexpr int PER = (HALF + 31) / 32;
      int32_t my_slot[PER];
      float my_w[PER];
      if (!g1 && args.ksplit <= 1) {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int t = t_begin + j * 32 + lane;
          my_slot[j] = 0;
          my_w[j] = 0.f;
          if (t < t_end && t < item.rows_t) {
            const int64_t p = static_cast<int64_t>(item.row0) + t;
            my_slot[j] = args.sorted_slots != nullptr ? args.sorted_slots[p] : static_cast<int32_t>(p);
            my_w[j] = args.topk_w != nullptr ? args.topk_w[my_slot[j]] : 1.f;
          }
        }
      }
      // one token's outputs from the two fp32 accumulators of row r (tl: token within
      // this warp's share; warp-uniform, so the early return keeps the warp converged)
      auto emit = [&](int tl, float a0, float a1) {
        const int t = t_begin + tl;
        if (t >= t_end || t >= item.rows_t) return;
        const int64_t p = static_cast<int64_t>(item.row0) + t;
        if (g1) {
          const float g = round_bf16(a0);
          const float up = round_bf16(a1);
          const float silu = round_bf16(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))));
          const int n = item.rb * ROWS + r;
          const int pos = FAST ? kperm_pos(n) : n;
          P.out[p * P.n_out + pos] = __float2bfloat16_rn(__fmul_rn(silu, up));
        } else {
          if (args.ksplit > 1) {  // fp32 partial of this K slice, summed in order by splitk_reduce
            float* prow = args.partial + (static_cast<int64_t>(item.ks) * args.dense_rows + p) * P.n_out +
                          item.rb * 2 * ROWS + r;
            prow[0] = a0;
            prow[ROWS] = a1;
            return;
          }
          const int32_t slot = __shfl_sync(0xffffffffu, my_slot[tl >> 5], tl & 31);
          const float w = __shfl_sync(0xffffffffu, my_w[tl >> 5], tl & 31);
          __nv_bfloat16* orow;
          if (args.ep_on) {
            const int src = slot / args.ep.L.cap;
            const int64_t at = static_cast<int64_t>(args.ep.me) * args.ep.L.cap + (slot - src * args.ep.L.cap);
            orow = reinterpret_cast<__nv_bfloat16*>(args.ep.peers[src] + args.ep.L.back) + at * P.n_out;
          } else {
            orow = P.out + static_cast<int64_t>(slot) * P.n_out;
          }
          orow += item.rb * 2 * ROWS + r;
          orow[0] = __float2bfloat16_rn(__fmul_rn(a0, w));
          orow[ROWS] = __float2bfloat16_rn(__fmul_rn(a1, w));
        }
      };
      if (FAST) {
        const int sbuf = ii & 1;
        float acc0[FAST ? HALF : 1], acc1[FAST ? HALF : 1];
#pragma unroll
        for (int i = 0; i < (FAST ? HALF : 1); ++i) acc0[i] = acc1[i] = 0.f;
        if (!mbar_wait(&sc_full[sbuf], (ii >> 1) & 1, abort_flag, 0x400)) break;
        const float* s0row = ssc + sbuf * (2 * ROWS * MAX_G) + r * P.groups;
        const float* s1row = s0row + ROWS * MAX_G;
        for (int kc = 0; kc < P.K / KC; ++kc, ++it) {
          const int pb = it & 1;
          if (!mbar_wait(&mdone[it % BS], (it / BS) & 1, abort_flag, 0x410 + pb)) { ok = false; break; }
          tc_fence_after();
          const int gi = P.group > 0 ? (kc * KC) / P.group : 0;
          const float s0 = s0row[gi], s1 = s1row[gi];
          const uint32_t p0 = tmem + lane_addr + pb * 2 * NTM + t_begin, p1 = p0 + NTM;
#pragma unroll
          for (int c = 0; c < HALF / 8; ++c) {
            const int t0 = c * 8;
            if (t_begin + t0 < t_end) {
              float v0[8], v1[8];
              tc_ld8(p0 + t0, v0);
              tc_ld8(p1 + t0, v1);
              tc_wait_ld();  // one TMEM round trip for both tiles' columns
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                acc0[(c * 8 + i) % (FAST ? HALF : 1)] = __fmaf_rn(s0, v0[i], acc0[(c * 8 + i) % (FAST ? HALF : 1)]);
                acc1[(c * 8 + i) % (FAST ? HALF : 1)] = __fmaf_rn(s1, v1[i], acc1[(c * 8 + i) % (FAST ? HALF : 1)]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[pb]);
        }
        if (!ok) break;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // scale reads before the bulk refill
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_empty[sbuf]);
#pragma unroll
        for (int i = 0; i < (FAST ? HALF : 1); ++i) emit(i, acc0[i], acc1[i]);
      } else {
        const int ab = C::ACC_BUFS == 2 ? (ii & 1) : 0;
        const uint32_t ph = C::ACC_BUFS == 2 ? ((ii >> 1) & 1) : (ii & 1);
        const uint32_t acc_base = tmem + ab * C::ACC_BUF_COLS;
        if (!mbar_wait(&acc_full[ab], ph, abort_flag, 0x420)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HALF / 16; ++c) {
          const int t0 = t_begin + c * 16;
          if (t0 < t_end) {
            float v0[16], v1[16];
            tc_ld16(acc_base + lane_addr + t0, v0);
            tc_ld16(acc_base + lane_addr + SPLIT * NTM + t0, v1);
            if (SPLIT == 2) {
              float w0[16], w1[16];
              tc_ld16(acc_base + lane_addr + NTM + t0, w0);
              tc_ld16(acc_base + lane_addr + 3 * NTM + t0, w1);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                v0[i] = __fadd_rn(v0[i], w0[i]);
                v1[i] = __fadd_rn(v1[i], w1[i]);
              }
            } else {
              tc_wait_ld();
            }
            if (NTM >= 128 && g1 && args.ksplit <= 1) {
              // GEMM1 of 128-token tiles: silu(gate) * up for 16 tokens as straight-line
              // code (the exp of all 16 first, then the divisions, then the stores) so
              // that the chains overlap (measured with 8 experts x 256 rows: fused launch
              // 82 -> 72 us; the 64-token tiles, whose epilogue overlaps the next item's
              // MMAs, keep the per-token form: 117 vs 119 us at C3)
              float e[16], o[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                v0[i] = round_bf16(v0[i]);
                e[i] = __fadd_rn(1.f, expf(-v0[i]));
              }
              uint32_t slow = 0;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                bool need;
                o[i] = silu_quot_fast(v0[i], e[i], need);
                slow |= static_cast<uint32_t>(need) << i;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __fmul_rn(round_bf16(o[i]), round_bf16(v1[i]));
              const TcPhase& P1 = args.ph[item.ph];
              const int n = item.rb * ROWS + r;
              __nv_bfloat16* col = P1.out + (FAST ? kperm_pos(n) : n);
              const int tl0 = t_begin + c * 16;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int t = tl0 + i;
                if (t < t_end && t < item.rows_t)
                  col[(static_cast<int64_t>(item.row0) + t) * P1.n_out] = __float2bfloat16_rn(o[i]);
              }
              // rare (quotients near a bf16 rounding midpoint): those tokens again from the
              // accumulators, still in TMEM, with the IEEE division, stored over the fast
              // values.  Kept after the stores so that the common path holds no extra
              // values live (a fallback inside it made the launch 9 us slower).
              if (__any_sync(0xffffffffu, slow != 0)) {
                static_assert(SPLIT == 1, "the fallback reloads one accumulator per tile");
                float w0[16], w1[16];
                tc_ld16(acc_base + lane_addr + t0, w0);
                tc_ld16(acc_base + lane_addr + SPLIT * NTM + t0, w1);
                tc_wait_ld();
#pragma unroll 1
                for (int i = 0; i < 16; ++i) {
                  const int t = tl0 + i;
                  if (((slow >> i) & 1u) && t < t_end && t < item.rows_t) {
                    const float g = round_bf16(w0[i]);
                    const float q = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
                    col[(static_cast<int64_t>(item.row0) + t) * P1.n_out] =
                        __float2bfloat16_rn(__fmul_rn(round_bf16(q), round_bf16(w1[i])));
                  }
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) emit(c * 16 + i, v0[i], v1[i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
      }
      if (args.fused && item.ph == 0) {
        // this warp's rows of h are stored: count it for the token tile's GEMM2 items
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(args.tile_done + item.tg, 1);
      }
    }
  }

  if ((!GEMM1 || args.fused) && args.ep_on && warp >= FIRST_EPI) __threadfence_system();  // rows stored to peers
  tc_fence_before();
  __syncthreads();
  pdl_trigger();
  if (args.fused && threadIdx.x == 0) {
    // the last CTA out leaves the tile counters zeroed for the next launch
    int* cta_done = args.tile_done + args.tile_done_n;
    __threadfence();
    if (atomicAdd(cta_done, 1) == static_cast<int>(gridDim.x) - 1) {
      for (int i = 0; i < args.tile_done_n; ++i) args.tile_done[i] = 0;
      __threadfence();
      atomicExch(cta_done, 0);
    }
  }
  if (warp == FIRST_MMA) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if ((!GEMM1 || args.fused) && args.ep_on && threadIdx.x == 0) {
    // last CTA out tells every source rank that its rows are back
    if (atomicAdd(args.ep.done, 1u) == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < args.ep.L.R; ++d)
        st_release_sys(ep_sig(args.ep.peers[d], args.ep.L, kEpRflag) + args.ep.me, args.ep.epoch);
      atomicExch(args.ep.done, 0u);
    }
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

template <int BITS, int NTM>
int phase_maps(const void* act, int64_t n_rows, int K, int E, int rows_total, const int8_t* q, CUtensorMap* tw,
               CUtensorMap* tb) {
  const uint64_t k_bytes = static_cast<uint64_t>(K) * BITS / 8;
  int rc = BITS == 16 ? make_map(tw, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, static_cast<uint64_t>(E) * rows_total,
                                 k_bytes, 64, ROWS, CU_TENSOR_MAP_SWIZZLE_128B)
                      : make_map(tw, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_bytes, static_cast<uint64_t>(E) * rows_total,
                                 k_bytes, 128, ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  for (int i = 0; i < 4; ++i) {
    const uint32_t box = 16u << (i < 3 || NTM >= 128 ? i : 2);
    rc = make_map(&tb[i], act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, static_cast<uint64_t>(n_rows),
                  static_cast<uint64_t>(K) * 2, 64, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  return LLQ_OK;
}

inline TcPhase make_phase(bool gemm1, const float* scale, void* out, int K, int rows_total, int inter, int n_out,
                          int group_size) {
  TcPhase P;
  P.scale = scale;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.K = K;
  P.rows_total = rows_total;
  P.inter = inter;
  P.n_out = n_out;
  P.rblocks = gemm1 ? inter / ROWS : n_out / (2 * ROWS);
  const bool grouped = group_size > 0 && K % group_size == 0;
  P.group = grouped ? group_size : 0;
  P.groups = grouped ? K / group_size : 1;
  return P;
}

template <bool GEMM1, int BITS, bool FAST, int NTM>
int launch_kernel(const CUtensorMap (&tw)[2], const CUtensorMap (&tb)[2][4], const TcArgs& a, cudaStream_t st) {
  using C = Cfg<GEMM1, BITS, FAST, NTM>;
  static std::atomic<uint64_t> attr{0};
  if (first_use_on_device(attr))
    cudaFuncSetAttribute(moe_gemm_tc_kernel<GEMM1, BITS, FAST, NTM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(C::SMEM_BYTES));
  // one CTA per SM; a fused launch's GEMM2 items wait for other CTAs' GEMM1 items, so it
  // is launched cooperatively and fails at launch where its grid cannot be co-resident
  launch_pdl_ex(a.fused != 0, moe_gemm_tc_kernel<GEMM1, BITS, FAST, NTM>, dim3(num_sms()), dim3(C::THREADS),
                C::SMEM_BYTES, st, tw[0], tb[0][0], tb[0][1], tb[0][2], tb[0][3], tw[1], tb[1][0], tb[1][1],
                tb[1][2], tb[1][3], a);
  return check_launch("moe_gemm_tc_kernel");
}

template <bool GEMM1, int BITS, bool FAST, int NTM>
int launch_tc(const void* act, int64_t n_rows, const int32_t* offsets, int E, int K, int rows_total,
              int inter, int n_out, const int8_t* q, const float* scale, int group_size,
              const int32_t* sorted_slots, const float* topk_w, void* out, cudaStream_t st,
              const EpScatter* ep, int ksplit = 1, float* partial = nullptr) {
  if (n_rows <= 0) return LLQ_OK;
  CUtensorMap tw[2], tb[2][4];
  int rc = phase_maps<BITS, NTM>(act, n_rows, K, E, rows_total, q, &tw[0], tb[0]);
  if (rc) return rc;
  tw[1] = tw[0];
  for (int i = 0; i < 4; ++i) tb[1][i] = tb[0][i];
  TcArgs a{};
  a.offsets = offsets;
  a.dense_rows = offsets == nullptr ? static_cast<int>(n_rows) : 0;
  a.ksplit = ksplit;
  a.partial = partial;
  a.sorted_slots = sorted_slots;
  a.topk_w = topk_w;
  a.E = E;
  a.ph[0] = make_phase(GEMM1, scale, out, K, rows_total, inter, n_out, group_size);
  a.ph[1] = a.ph[0];
  a.fused = 0;
  a.tile_done = nullptr;
  a.ep_on = ep != nullptr;
  if (ep != nullptr) a.ep = *ep;
  return launch_kernel<GEMM1, BITS, FAST, NTM>(tw, tb, a, st);
}

// GEMM1 and GEMM2 of one layer in one persistent launch (exact mode): GEMM2 items
// follow the GEMM1 items and start as soon as their token tile's h rows are stored
template <int BITS, int NTM, bool FAST = false>
int launch_fused(const void* x_sorted, void* h_sorted, int64_t n_rows, const int32_t* offsets, int E, int H, int I,
                 const int8_t* qw1, const float* sw1, const int8_t* qw2, const float* sw2, int group_size,
                 const int32_t* sorted_slots, const float* topk_w, void* y_slots, int* tile_done,
                 int tile_done_n, cudaStream_t st, const EpScatter* ep) {
  if (n_rows <= 0) return LLQ_OK;
  CUtensorMap tw[2], tb[2][4];
  int rc = phase_maps<BITS, NTM>(x_sorted, n_rows, H, E, 2 * I, qw1, &tw[0], tb[0]);
  if (rc) return rc;
  rc = phase_maps<BITS, NTM>(h_sorted, n_rows, I, E, H, qw2, &tw[1], tb[1]);
  if (rc) return rc;
  TcArgs a{};
  a.offsets = offsets;
  a.dense_rows = 0;
  a.ksplit = 1;
  a.partial = nullptr;
  a.sorted_slots = sorted_slots;
  a.topk_w = topk_w;
  a.E = E;
  a.ph[0] = make_phase(true, sw1, h_sorted, H, 2 * I, I, I, group_size);
  a.ph[1] = make_phase(false, sw2, y_slots, I, H, 0, H, group_size);
  a.fused = 1;
  a.tile_done = tile_done;
  a.tile_done_n = tile_done_n;
  a.ep_on = ep != nullptr;  // GEMM2 rows go to the source ranks' windows
  if (ep != nullptr) a.ep = *ep;
  return launch_kernel<true, BITS, FAST, NTM>(tw, tb, a, st);
}

// decode tiles (64 tokens) unless the average expert holds more than 96 rows
// (rows_hint: the expected number of rows, when n_rows is a capacity)
template <bool GEMM1, int BITS, bool FAST>
int launch_any(int64_t n_rows, int E, const void* act, const int32_t* offsets, int K, int rows_total,
               int inter, int n_out, const int8_t* q, const float* scale, int group_size,
               const int32_t* sorted_slots, const float* topk_w, void* out, cudaStream_t st,
               int64_t rows_hint, const EpScatter* ep) {
  if (!FAST && rows_hint > static_cast<int64_t>(E) * 96)
    return launch_tc<GEMM1, BITS, false, 128>(act, n_rows, offsets, E, K, rows_total, inter, n_out, q, scale,
                                              group_size, sorted_slots, topk_w, out, st, ep);
  return launch_tc<GEMM1, BITS, FAST, 64>(act, n_rows, offsets, E, K, rows_total, inter, n_out, q, scale,
                                          group_size, sorted_slots, topk_w, out, st, ep);
}

// out[m, n] = bf16(sum over slices s, in order, of partial[s][m][n])
__global__ void splitk_reduce_kernel(const float4* __restrict__ partial, int ksplit, int64_t n4,
                                     uint2* __restrict__ out) {
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = __ldg(partial + i);
    for (int s = 1; s < ksplit; ++s) {
      const float4 v = __ldg(partial + static_cast<int64_t>(s) * n4 + i);
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    out[i] = o;
  }
}

template <int BITS, int NTM>
int dense_tc(const void* x, int64_t M, int K, int N, const int8_t* q, const float* scale, int group_size, void* out,
             int ksplit, float* partial, cudaStream_t st) {
  int rc = launch_tc<false, BITS, false, NTM>(x, M, nullptr, 1, K, N, 0, N, q, scale, group_size, nullptr, nullptr,
                                              out, st, nullptr, ksplit, partial);
  if (rc || ksplit == 1) return rc;
  const int64_t n4 = M * N / 4;
  int64_t blocks = (n4 + 255) / 256;
  if (blocks > static_cast<int64_t>(num_sms()) * 8) blocks = static_cast<int64_t>(num_sms()) * 8;
  launch_pdl(splitk_reduce_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
             reinterpret_cast<const float4*>(partial), ksplit, n4, static_cast<uint2*>(out));
  return check_launch("splitk_reduce_kernel");
}

}  // namespace

bool tc_supported(int E, int N_out, int K, int bits, int group_size, bool gemm1) {
  if (bits != 4 && bits != 8) return false;
  if (E < 1 || E > MAX_E) return false;
  if (K % KC != 0 || K > KC * MAX_G) return false;
  if (N_out % (gemm1 ? ROWS : 2 * ROWS) != 0) return false;
  const bool grouped = group_size > 0 && K % group_size == 0;
  if (grouped && group_size % KC != 0) return false;  // one scale per 128-element step
  return true;
}

int gemm1_tc(const void* x_sorted, const int32_t* offsets, int64_t n_rows, int E, int H, int I,
             const int8_t* qw1, const float* sw1, int bits, int group_size, void* h_sorted, bool fast,
             cudaStream_t st, int64_t rows_hint) {
  if (!tc_supported(E, I, H, bits, group_size, true))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM1: unsupported shape");
  if (fast && bits != 4) return fail(LLQ_EUNSUPPORTED, "fast dequantization is INT4 only");
  if (rows_hint < 0) rows_hint = n_rows;
  if (bits == 4) {
    if (fast)
      return launch_any<true, 4, true>(n_rows, E, x_sorted, offsets, H, 2 * I, I, I, qw1, sw1, group_size,
                                       nullptr, nullptr, h_sorted, st, rows_hint, nullptr);
    return launch_any<true, 4, false>(n_rows, E, x_sorted, offsets, H, 2 * I, I, I, qw1, sw1, group_size,
                                      nullptr, nullptr, h_sorted, st, rows_hint, nullptr);
  }
  return launch_any<true, 8, false>(n_rows, E, x_sorted, offsets, H, 2 * I, I, I, qw1, sw1, group_size,
                                    nullptr, nullptr, h_sorted, st, rows_hint, nullptr);
}

int gemm2_tc(const void* h_sorted, const int32_t* offsets, const int32_t* sorted_slots,
             const float* topk_w, int64_t n_rows, int E, int H, int I, const int8_t* qw2,
             const float* sw2, int bits, int group_size, void* y_slots, bool fast, cudaStream_t st,
             int64_t rows_hint, const EpScatter* ep) {
  if (!tc_supported(E, H, I, bits, group_size, false))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM2: unsupported shape");
  if (fast && bits != 4) return fail(LLQ_EUNSUPPORTED, "fast dequantization is INT4 only");
  if (rows_hint < 0) rows_hint = n_rows;
  if (bits == 4) {
    if (fast)
      return launch_any<false, 4, true>(n_rows, E, h_sorted, offsets, I, H, 0, H, qw2, sw2, group_size,
                                        sorted_slots, topk_w, y_slots, st, rows_hint, ep);
    return launch_any<false, 4, false>(n_rows, E, h_sorted, offsets, I, H, 0, H, qw2, sw2, group_size,
                                       sorted_slots, topk_w, y_slots, st, rows_hint, ep);
  }
  return launch_any<false, 8, false>(n_rows, E, h_sorted, offsets, I, H, 0, H, qw2, sw2, group_size,
                                     sorted_slots, topk_w, y_slots, st, rows_hint, ep);
}

// token tiles are >= 64 rows, plus one partial tile per expert; one more slot counts CTAs
int gemm12_counter_slots(int64_t n_rows, int E) { return static_cast<int>(n_rows / 16 + E + 2); }

// GEMM1 + GEMM2 over bf16 weights dequantized beforehand (prefill-sized batches, where
// each weight meets many token tiles): TMA brings both operands to shared memory and
// the kernel's warps only load, multiply and run the epilogues
int gemm12_fused_bf16_tc(const void* x_sorted, const int32_t* offsets, const int32_t* sorted_slots,
                         const float* topk_w, int64_t n_rows, int E, int H, int I, const void* w1, const void* w2,
                         void* h_sorted, void* y_slots, int* tile_done, cudaStream_t st, const EpScatter* ep) {
  if (E < 1 || E > MAX_E || H % KC != 0 || I % KC != 0 || H > KC * MAX_G || I > KC * MAX_G || H % (2 * ROWS) != 0)
    return fail(LLQ_EUNSUPPORTED, "tcgen05 bf16 expert GEMMs: unsupported shape");
  const int tile_done_n = gemm12_counter_slots(n_rows, E) - 1;
  return launch_fused<16, 128>(x_sorted, h_sorted, n_rows, offsets, E, H, I, static_cast<const int8_t*>(w1), nullptr,
                               static_cast<const int8_t*>(w2), nullptr, 0, sorted_slots, topk_w, y_slots, tile_done,
                               tile_done_n, st, ep);
}


int gemm12_fused_tc(const void* x_sorted, const int32_t* offsets, const int32_t* sorted_slots, const float* topk_w,
                    int64_t n_rows, int E, int H, int I, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                    const float* sw2, int bits, int group_size, void* h_sorted, void* y_slots, int* tile_done,
                    cudaStream_t st, int64_t rows_hint, const EpScatter* ep, bool fast) {
  if (!tc_supported(E, I, H, bits, group_size, true) || !tc_supported(E, H, I, bits, group_size, false))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 expert GEMMs: unsupported shape");
  const int tile_done_n = gemm12_counter_slots(n_rows, E) - 1;
  if (fast) {  // scale-after-MMA mode: INT4, 64-token tiles (token rows K-interleaved by the permute)
    if (bits != 4) return fail(LLQ_EUNSUPPORTED, "fast dequantization is INT4 only");
    return launch_fused<4, 64, true>(x_sorted, h_sorted, n_rows, offsets, E, H, I, qw1, sw1, qw2, sw2, group_size,
                                     sorted_slots, topk_w, y_slots, tile_done, tile_done_n, st, ep);
  }
  if (rows_hint < 0) rows_hint = n_rows;
  const bool wide = rows_hint > static_cast<int64_t>(E) * 96;
  if (bits == 4)
    return wide ? launch_fused<4, 128>(x_sorted, h_sorted, n_rows, offsets, E, H, I, qw1, sw1, qw2, sw2, group_size,
                                       sorted_slots, topk_w, y_slots, tile_done, tile_done_n, st, ep)
                : launch_fused<4, 64>(x_sorted, h_sorted, n_rows, offsets, E, H, I, qw1, sw1, qw2, sw2, group_size,
                                      sorted_slots, topk_w, y_slots, tile_done, tile_done_n, st, ep);
  return wide ? launch_fused<8, 128>(x_sorted, h_sorted, n_rows, offsets, E, H, I, qw1, sw1, qw2, sw2, group_size,
                                     sorted_slots, topk_w, y_slots, tile_done, tile_done_n, st, ep)
              : launch_fused<8, 64>(x_sorted, h_sorted, n_rows, offsets, E, H, I, qw1, sw1, qw2, sw2, group_size,
                                    sorted_slots, topk_w, y_slots, tile_done, tile_done_n, st, ep);
}

}  // namespace llq


namespace llq {

// A dense layer takes 128-token tiles only above this many rows: up to it, 64-token tiles
// keep the deeper weight ring, and the tiles sharing a weight block read it from L2
constexpr int64_t kDenseWideRows = 128;

// K slices for a dense layer: enough work items to cover the SMs, each slice a
// whole number of 128-wide K steps
int dense_ksplit(int64_t M, int K, int N) {
  const int ntm = M > kDenseWideRows ? 128 : 64;
  const int64_t items = (M + ntm - 1) / ntm * (N / (2 * ROWS));
  const int kch = K / KC;
  int ks = 1;
  while (items * ks * 2 <= num_sms() && kch % (ks * 2) == 0) ks *= 2;
  return ks;
}

int dense_linear_tc(const void* x, int64_t M, int K, int N, const int8_t* q, const float* scale, int bits,
                    int group_size, void* out, void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (!tc_supported(1, N, K, bits, group_size, false))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 dense linear needs K %% 128 == 0, K <= 2048, N %% 256 == 0 and "
                                  "group %% 128 == 0 (K=%d N=%d group=%d)", K, N, group_size);
  const int ks = dense_ksplit(M, K, N);
  const size_t need = ks > 1 ? static_cast<size_t>(ks) * M * N * 4 : 0;
  if (ks > 1 && (workspace == nullptr || ws_bytes < need))
    return fail(LLQ_ENOSPACE, "quant_linear workspace needs %zu bytes, got %zu", need, ws_bytes);
  float* partial = static_cast<float*>(workspace);
  if (M > kDenseWideRows) {
    return bits == 4 ? dense_tc<4, 128>(x, M, K, N, q, scale, group_size, out, ks, partial, st)
                     : dense_tc<8, 128>(x, M, K, N, q, scale, group_size, out, ks, partial, st);
  }
  return bits == 4 ? dense_tc<4, 64>(x, M, K, N, q, scale, group_size, out, ks, partial, st)
                   : dense_tc<8, 64>(x, M, K, N, q, scale, group_size, out, ks, partial, st);
}

}  // namespace llq
