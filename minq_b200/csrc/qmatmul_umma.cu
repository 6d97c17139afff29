// Batched quantized projections on the 5th-generation tensor cores:
// Y[b] = W X[b] for Q4_0 / Q8_0 weights (quantize.rs:215-280, the
// reference's QuantizedTensor::matvec run once per sequence) and 1..64
// inputs, with tcgen05.mma accumulating in tensor memory (TMEM). The input
// RMSNorm (tensor.rs:219-227) is applied while the inputs are prepared;
// bias / residual / SwiGLU are applied after the sum.
//
// Operands. A = weight codes of 128 rows as exact bf16 (Q4_0: nibble - 8,
// Q8_0: the i8 code), held in TMEM (lane = row, two bf16 per column);
// B = the inputs split into x_hi = bf16(x) and x_lo = bf16(x - x_hi) in
// shared memory: both parts accumulate into the same TMEM tile, so a
// block's sum_k code_k x_k carries the input to 2^-18 of |x| (16
// significand bits of the split, then f32 accumulation). The block scale d
// multiplies each 32-column block's sum once, in block order, into the
// row's running f32 sum (acc += d * sum, quantize.rs:252-280), so every
// block gets its own accumulator in TMEM and an epilogue pass. Q4_0 codes
// are unpacked in the column order 0, 4, 1, 5, 2, 6, 3, 7 of each 8-column
// group (two lop3 / one bf16 subtraction per pair) and the inputs are
// written in the same order; the sum over k does not depend on it.
//
// Data flow in one CTA (128 weight rows -- 64 + 64 for gate and up -- by
// one K slice, in chunks of 4 blocks = 128 columns through a ring of S
// shared-memory stages):
//   warp 0           TMA, one elected lane: per chunk the raw weight rows (a
//                    2-D box of the row-major block stream, no swizzle,
//                    evict-first) and the four 64-column x_hi / x_lo tiles
//                    (128-byte swizzle; x_hi rows then x_lo rows, each
//                    half a B operand of N = NP); warp 0 also owns the
//                    TMEM allocation
//   warps 1, 2       tcgen05.mma issue, one lane each: warp 1 blocks 0-1 of
//                    every chunk, warp 2 blocks 2-3. A comes from TMEM (the
//                    chunk's A tile), B from the stage; block g accumulates
//                    in TMEM set g mod NBUF with four MMAs (two k steps,
//                    x_hi and x_lo into the same columns), then
//                    tcgen05.commit to that set's barrier
//   4 unpacker warps thread = weight row (TMEM lane): the chunk's codes ->
//                    exact bf16 with lop3 / one bf16 subtraction per pair,
//                    tcgen05.st into A tile (chunk mod 2)
//   4 WG epilogue    thread = weight row and CW inputs: tcgen05.ld of each
//   warps            block's sums, release of the set, then acc += d * sum
//                    in block order; at the end bias / residual / SwiGLU
//                    and the store (or the slice partial)
// The K range splits into S slices (a wave cost model picks S; row tiles
// that overrun whole waves go to a second launch) whose partials
// um_reduce_kernel sums in slice order.
// Every mbarrier wait is time-bounded (1 s); a timeout sets the device
// status word and an abort flag that ends every role's loop, after which
// the producer waits for its copies in flight, the MMA threads for their
// MMAs, and warp 0 frees the TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "matvec_common.cuh"
#include "pipeline.cuh"

namespace minq {

namespace {

constexpr int kUmChunkBlocks = 4;  // blocks per staged chunk (128 columns)
constexpr int kUmCtrlWarps = 4;    // warp 0 producer / TMEM, warps 1-2 MMA issue (warp 3 idle)
constexpr int kUmMaxStages = 6;
constexpr int kUmIssuers = 2;      // MMA-issuing warps (1, 2): blocks 0-1 and 2-3 of each chunk
constexpr size_t kUmSmemLimit = 227 * 1024;

constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// NP: inputs padded to 16 / 32 / 64. The stage holds x_hi and x_lo of the NP
// inputs as 2 NP rows; each part is the B operand (N = NP) of its own MMA
// into the same accumulator columns. (Stacking both as one MMA of N = 2 NP
// costs less tensor time -- a kind::f16 MMA takes ~51 cycles for any N <= 64,
// 64 at N = 128 -- but doubles the columns of an accumulator set and so
// halves the sets in flight; the tensor pipe is not what bounds the kernel.)
template <int DT, int NP>
struct UmGeom {
  static constexpr int ROWS = 128;                            // weight rows per CTA
  static constexpr int NN = 2 * NP;                           // MMA N: x_hi rows, then x_lo rows
  static constexpr int bb = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  static constexpr int raw_pitch = kUmChunkBlocks * bb;       // bytes of one row of a raw chunk
  static constexpr int raw_bytes = ROWS * raw_pitch;
  static constexpr int xsub_bytes = NN * 128;                 // one 64-column half: hi rows, lo rows
  static constexpr int x_bytes = 2 * xsub_bytes;
  static constexpr int stage_bytes = (x_bytes + raw_bytes + 1023) & ~1023;
  static constexpr int WG = NP == 64 ? 4 : 2;                 // epilogue warps per TMEM lane quarter
  static constexpr int CW = NP / WG;                          // inputs summed per epilogue thread
  static constexpr int UNP = 4;                               // unpacker warps (one per lane quarter)
  static constexpr int EPI = 4 * WG;                          // epilogue warps
  static constexpr int WARPS = kUmCtrlWarps + UNP + EPI;
  static constexpr int THREADS = 32 * WARPS;
  // x_hi and x_lo accumulate into the same TMEM columns (two MMAs of N = NP
  // per k step): an accumulator set is NP columns, so up to 8 sets rotate
  // between the MMA issuers and the epilogue (measured against one MMA of
  // N = 2 NP into 2 NP columns with 3-4 sets: LLaMA-3-8B x 64 batched step
  // 10.05 -> 8.38 ms, Qwen3-4B 2048-token prefill 10030 -> 11560 tok/s)
  static constexpr int NACC = NP;                             // TMEM columns of one accumulator set
  static constexpr int NBUF = (384 / NACC) < 8 ? 384 / NACC : 8;  // sets (block g: set g mod NBUF)
  static constexpr int ACC_COLS = NBUF * NACC;                // TMEM columns of the accumulators
  static constexpr int A_COL0 = ACC_COLS;                     // A tiles: 2 chunks x 4 blocks x 16 columns
  static constexpr int TMEM_COLS = pow2_at_least(A_COL0 + 128);
  // dynamic shared memory for S stages: alignment slack, ring, barriers
  static constexpr size_t smem(int S) { return 1024 + (size_t)S * stage_bytes + 512; }
  static constexpr int max_stages() {
    int s = kUmMaxStages;
    while (s > 2 && smem(s) > kUmSmemLimit) --s;
    return s;
  }
};

struct UmParams {
  size_t rows;      // rows of each matrix
  int B;
  int S;            // column slices
  int slice_chunks; // chunks per slice
  int nchunks;      // chunks of the whole row
  int stages;
  const float* bias;      // [rows] or null
  const float* residual;  // [B][y_stride] or null (may alias y)
  float* y;               // [B][y_stride]
  size_t y_stride;
  float* part;            // S > 1: [S][halves][B][rows]
  int tile0;              // first row tile of the launch (blockIdx.x + tile0)
  size_t row0, nrows;     // rows the reduce kernel finishes (S > 1)
  int* status;
};

// ---------------------------------------------------------------------------
// tcgen05 / TMEM building blocks (inline PTX, sm_100a)

__device__ __forceinline__ void tc05_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc05_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte
// offset), descriptor version 1, layout type 2 (SWIZZLE_128B). The start
// address may sit 32 / 64 / 96 bytes into the swizzle row to select a
// 16-column k step; the 8-row group it belongs to must be 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D f32, A and B bf16, both K-major,
// M = 128, N columns.
template <int N>
__device__ __forceinline__ constexpr uint32_t um_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D (TMEM) (+)= A (TMEM, 128 lanes x 16 bf16) x B (shared memory descriptor).
__device__ __forceinline__ void umma_bf16_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(dtmem),
      "r"(atmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The mbarrier tracks completion of every tcgen05 operation this thread
// issued before (one arrival when they are done).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 8 / 16 columns of f32 from TMEM (lane quarter of this warp).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Wait for this thread's TMEM loads; the registers pass through the asm so
// no use of them can be scheduled before the wait.
template <int K>
__device__ __forceinline__ void tmem_wait_ld(uint32_t* r) {
  static_assert(K == 8 || K == 16 || K == 32, "");
  if constexpr (K == 8) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
  } else if constexpr (K == 16) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
  } else {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
  }
}

// 32 lanes x 32 columns into TMEM (lane quarter of this warp); completion
// is awaited with tcgen05.wait::st.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}


__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t u) {
  __nv_bfloat162 v;
  memcpy(&v, &u, 4);
  return v;
}

// The 8 codes of a Q4_0 code word w (nibble i = column i of its 8-column
// group) as exact bf16 (code - 8), in the order 0, 4, 1, 5, 2, 6, 3, 7:
// (w >> 4j) & 0x000F000F | 0x43004300 holds bf16(128 + nibble j) and
// bf16(128 + nibble j + 4); subtracting bf16(136) = 0x4308 leaves code - 8.
__device__ __forceinline__ void q4_word_bf16(uint32_t w, uint32_t* o) {
  const __nv_bfloat162 off = bits_bf2(0x43084308u);
  o[0] = bf2_bits(__hsub2(bits_bf2((w & 0x000F000Fu) | 0x43004300u), off));
  o[1] = bf2_bits(__hsub2(bits_bf2(((w >> 4) & 0x000F000Fu) | 0x43004300u), off));
  o[2] = bf2_bits(__hsub2(bits_bf2(((w >> 8) & 0x000F000Fu) | 0x43004300u), off));
  o[3] = bf2_bits(__hsub2(bits_bf2(((w >> 12) & 0x000F000Fu) | 0x43004300u), off));
}

// Codes (bytes) e, e + 1 of a Q8_0 code word as exact bf16.
__device__ __forceinline__ uint32_t q8_pair_bf16(uint32_t w, int e) {
  const float a = (float)(int8_t)((w >> (8 * e)) & 0xFFu);
  const float b = (float)(int8_t)((w >> (8 * e + 8)) & 0xFFu);
  return bf2_bits(__floats2bfloat162_rn(a, b));
}

// Bounded mbarrier wait shared by every role: returns false once the abort
// flag is set (by any thread) or after 1 s, when it sets the flag and the
// device status word.
__device__ __forceinline__ bool um_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      if (status) atomicOr(status, kDeviceTimeout);
      return false;
    }
  }
}

// One lane of a converged warp (elect.sync).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// The same for a whole warp: every lane waits, and the warp goes on only
// if all of them saw the phase (an abort seen by one lane stops all).
__device__ __forceinline__ bool um_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                             int* status) {
  const bool ok = um_wait(bar, parity, abort, status);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------

// x[b] -> x_hi / x_lo (bf16), optionally RMSNorm'd first with the
// reference's f32 operations (x * inv * w). With `perm`, position p of each
// 8-column group holds column (0, 4, 1, 5, 2, 6, 3, 7)[p] (the order the Q4_0
// codes are unpacked in); else columns stay in place. CTA (b, j) writes
// columns [1024 j, 1024 j + 1024) of input b, eight per thread.
constexpr int kUmPrepCols = 1024;
__global__ void __launch_bounds__(128) um_xprep_kernel(const float* __restrict__ x, size_t x_stride,
                                                      int n, const float* __restrict__ w, float eps,
                                                      int perm, __nv_bfloat16* __restrict__ xh,
                                                      __nv_bfloat16* __restrict__ xl) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[5];
  const float* row = x + (size_t)blockIdx.x * x_stride;
  float inv = 1.0f;
  if (w) {
    float ss = 0.0f;
    const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
    for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) {
      const float4 v = r4[i];
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = 0.0f;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) v += red[k];
      red[4] = 1.0f / sqrtf(v / (float)n + eps);
    }
    __syncthreads();
    inv = red[4];
  }
  const int c = blockIdx.y * kUmPrepCols + 8 * threadIdx.x;
  if (c >= n) return;
  float v[8];
  *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(row + c);
  *reinterpret_cast<float4*>(v + 4) = *reinterpret_cast<const float4*>(row + c + 4);
  if (w) {
    float g[8];
    *reinterpret_cast<float4*>(g) = *reinterpret_cast<const float4*>(w + c);
    *reinterpret_cast<float4*>(g + 4) = *reinterpret_cast<const float4*>(w + c + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * g[i];
  }
  float o[8];
  if (perm) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = v[i];
      o[2 * i + 1] = v[i + 4];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[i];
  }
  uint4 hh, ll;
  uint32_t* hp = &hh.x;
  uint32_t* lp = &ll.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    const float2 f = __bfloat1622float2(h);
    hp[i] = bf2_bits(h);
    lp[i] = bf2_bits(__floats2bfloat162_rn(o[2 * i] - f.x, o[2 * i + 1] - f.y));
  }
  const size_t off = (size_t)blockIdx.x * n + c;
  *reinterpret_cast<uint4*>(xh + off) = hh;
  *reinterpret_cast<uint4*>(xl + off) = ll;
}

template <int DT, int NP, bool DUAL>
__global__ void __launch_bounds__(UmGeom<DT, NP>::THREADS, 1)
    qmm_umma_kernel(const __grid_constant__ CUtensorMap mw0, const __grid_constant__ CUtensorMap mw1,
                    const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl,
                    UmParams p) {
  using G = UmGeom<DT, NP>;
  constexpr int ROWS = G::ROWS, CW = G::CW;
  constexpr int HR = DUAL ? ROWS / 2 : ROWS;  // rows of each matrix in this CTA
  extern __shared__ unsigned char um_sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = p.stages;

  // shared memory: [align][stage 0..S-1: x tiles | raw][barriers]
  const uint32_t base = (smem_u32(um_sm) + 1023u) & ~1023u;
  unsigned char* gbase = um_sm + (base - smem_u32(um_sm));
  const uint32_t ring = base;
  unsigned char* ctl = gbase + (size_t)S * G::stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctl);
  uint64_t* empty = full + kUmMaxStages;
  uint64_t* afull = empty + kUmMaxStages;
  uint64_t* aempty = afull + 2;
  uint64_t* accfull = aempty + 2;
  uint64_t* accempty = accfull + 8;
  uint64_t* mma_done = accempty + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int slice = blockIdx.y;
  const int kc0 = slice * p.slice_chunks;
  const int nch = min(p.nchunks, kc0 + p.slice_chunks) - kc0;
  const size_t rb = (size_t)(blockIdx.x + p.tile0) * HR;  // first row of each matrix

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < S; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], kUmIssuers + G::UNP + G::EPI);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&afull[i], G::UNP);
        mbar_init(&aempty[i], kUmIssuers);
      }
      for (int i = 0; i < G::NBUF; ++i) {
        mbar_init(&accfull[i], 1);
        mbar_init(&accempty[i], G::EPI);
      }
      mbar_init(&mma_done[0], 1);
      mbar_init(&mma_done[1], 1);
      *abort = 0;
      mbar_fence_init();
      asm volatile("prefetch.tensormap [%0];" ::"l"(&mw0) : "memory");
      if (DUAL) asm volatile("prefetch.tensormap [%0];" ::"l"(&mw1) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&mxh) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&mxl) : "memory");
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(G::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc05_fence_before();
  __syncthreads();
  tc05_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    // ---------------- producer: the warp runs the loop converged, one
    // elected lane issues the copies. Stage: for each 64-column half, x_hi
    // of the NP inputs then x_lo (the B operand, 2 NP rows), then the raw
    // weight rows.
    const uint64_t pol = policy_evict_first();
    int issued = 0;
    for (int cl = 0; cl < nch; ++cl) {
      const int s = cl % S, w = cl / S;
      if (w >= 1 && !um_wait_warp(&empty[s], (uint32_t)((w - 1) & 1), abort, p.status)) break;
      if (elect_one()) {
        unsigned char* st = gbase + (size_t)s * G::stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(G::x_bytes + G::raw_bytes));
        const int kc = kc0 + cl;
#pragma unroll
        for (int sh = 0; sh < 2; ++sh)
#pragma unroll
          for (int part = 0; part < 2; ++part)
            tma_load_2d_nohint(st + sh * G::xsub_bytes + part * NP * 128, part ? &mxl : &mxh,
                               kc * 128 + sh * 64, 0, &full[s]);
        unsigned char* raw = st + G::x_bytes;
        tma_load_2d(raw, &mw0, kc * G::raw_pitch, (int)rb, &full[s], pol);
        if (DUAL) tma_load_2d(raw + HR * G::raw_pitch, &mw1, kc * G::raw_pitch, (int)rb, &full[s], pol);
      }
      __syncwarp();
      issued = cl + 1;
    }
    // copies still in flight land before the CTA may exit
    for (int cl = max(0, issued - S); cl < issued; ++cl)
      mbar_wait_timed(&full[cl % S], (uint32_t)((cl / S) & 1), p.status);
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issue: lane 0 of warp 1 issues blocks 0-1 of
    // every chunk, lane 0 of warp 2 blocks 2-3 (A tile cl mod 2; block g
    // accumulates in set g mod NBUF with four MMAs of N = NP: two k steps,
    // x_hi and x_lo).
    // A kind::f16 MMA of N <= 64 takes ~51 cycles in the tensor core, about
    // the latency of a handful of dependent instructions of one thread, so
    // two threads issue, and each keeps its per-block work to a barrier
    // test, two adds, the MMAs and the commit: descriptors are formed once
    // and the stage and its phase advance incrementally.
    const int hi = warp - 1;  // which pair of blocks
    if (lane == 0) {
      constexpr uint32_t idesc = um_idesc<NP>();
      const uint64_t bdesc0 = sw128_desc(ring) + (uint64_t)((uint32_t)(hi * G::xsub_bytes) >> 4);
      const uint32_t a_tm = tmem + (uint32_t)(G::A_COL0 + hi * 32);
      int s = 0;                  // stage of chunk cl
      uint32_t sphase = 0;        // parity of its full barrier
      int g = 2 * hi;             // block index of the next MMA pair
      bool ok = true;
      for (int cl = 0; cl < nch && ok; ++cl) {
        const int a = cl & 1;
        if (!um_wait(&full[s], sphase, abort, p.status)) break;
        if (!um_wait(&afull[a], (uint32_t)((cl >> 1) & 1), abort, p.status)) break;
        const uint64_t bs = bdesc0 + (uint64_t)((uint32_t)(s * G::stage_bytes) >> 4);
        const uint32_t as = a_tm + (uint32_t)(a * 64);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          // set t was last used by block g - NBUF (either issuer): wait
          // until that block's sums are read
          const int t = g % G::NBUF, vv = g / G::NBUF;
          if (vv >= 1 && !um_wait(&accempty[t], (uint32_t)((vv - 1) & 1), abort, p.status)) {
            ok = false;
            break;
          }
          tc05_fence_after();
          const uint32_t d = tmem + (uint32_t)(t * G::NACC);
          // x_lo rows start NP rows (NP * 128 bytes) after x_hi's
          constexpr uint32_t lo = (uint32_t)(NP * 128) >> 4;
          umma_bf16_ts(d, as + (uint32_t)(jj * 16), bs + (uint64_t)((jj * 64) >> 4), idesc, 0u);
          umma_bf16_ts(d, as + (uint32_t)(jj * 16), bs + (uint64_t)(((jj * 64) >> 4) + lo), idesc, 1u);
          umma_bf16_ts(d, as + (uint32_t)(jj * 16 + 8), bs + (uint64_t)((jj * 64 + 32) >> 4), idesc, 1u);
          umma_bf16_ts(d, as + (uint32_t)(jj * 16 + 8), bs + (uint64_t)(((jj * 64 + 32) >> 4) + lo),
                       idesc, 1u);
          umma_commit(&accfull[t]);
          g += jj == 0 ? 1 : 3;  // next block of this issuer (skip the other pair)
        }
        if (!ok) break;
        umma_commit(&aempty[a]);
        umma_commit(&empty[s]);
        if (++s == S) {
          s = 0;
          sphase ^= 1u;
        }
      }
      // every MMA issued has finished before the TMEM is freed
      umma_commit(&mma_done[hi]);
      mbar_wait_timed(&mma_done[hi], 0, p.status);
    }
  } else if (warp >= kUmCtrlWarps && warp < kUmCtrlWarps + G::UNP) {
    // ---------------- unpackers: thread = weight row (TMEM lane); each
    // chunk's 4 blocks of codes -> bf16 into A tile cl mod 2, two blocks per
    // TMEM store
    const int v = (warp & 3) * 32 + lane;
    const uint32_t lq = (uint32_t)((warp & 3) * 32) << 16;
    for (int cl = 0; cl < nch; ++cl) {
      const int s = cl % S, w = cl / S, a = cl & 1;
      if (!um_wait_warp(&full[s], (uint32_t)(w & 1), abort, p.status)) break;
      if (cl >= 2 && !um_wait_warp(&aempty[a], (uint32_t)(((cl >> 1) - 1) & 1), abort, p.status)) break;
      const uint32_t src = ring + (uint32_t)(s * G::stage_bytes + G::x_bytes + v * G::raw_pitch + 4);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t o[32];
        if (DT == MINQ_Q4_0) {
          uint32_t wd[8];
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) wd[4 * j + i] = lds_u32(src + (uint32_t)((2 * hh + j) * G::bb + 4 * i));
#pragma unroll
          for (int i = 0; i < 8; ++i) q4_word_bf16(wd[i], o + 4 * i);
        } else {
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t wd = lds_u32(src + (uint32_t)((2 * hh + j) * G::bb + 4 * i));
              o[16 * j + 2 * i] = q8_pair_bf16(wd, 0);
              o[16 * j + 2 * i + 1] = q8_pair_bf16(wd, 2);
            }
        }
        // the store reads its registers when issued; one wait covers both
        tmem_st32(tmem + lq + (uint32_t)(G::A_COL0 + a * 64 + hh * 32), o);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc05_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[a]);
        mbar_arrive(&empty[s]);
      }
    }
  } else if (warp >= kUmCtrlWarps + G::UNP) {
    // ---------------- epilogue: thread = weight row (TMEM lane), inputs
    // [u CW, u CW + CW): acc += d * (block sums of x_hi, x_lo)
    const int wi = warp - kUmCtrlWarps - G::UNP;
    const int q = warp & 3;
    const int u = wi >> 2;
    const int v = q * 32 + lane;
    const uint32_t lq = (uint32_t)(q * 32) << 16;
    constexpr int JB = 1;                    // blocks per epilogue step (2 measured no faster)
    float acc[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) acc[i] = 0.0f;
    bool ok = true;
    for (int cl = 0; cl < nch && ok; ++cl) {
      const int s = cl % S, w = cl / S;
      if (!um_wait_warp(&full[s], (uint32_t)(w & 1), abort, p.status)) { ok = false; break; }
      const uint32_t raw = ring + (uint32_t)(s * G::stage_bytes + G::x_bytes + v * G::raw_pitch);
      float dsc[kUmChunkBlocks];
#pragma unroll
      for (int j = 0; j < kUmChunkBlocks; ++j) dsc[j] = __uint_as_float(lds_u32(raw + (uint32_t)(j * G::bb)));
      // JB blocks per step: one wait each, all their TMEM loads, one
      // wait::ld, the releases, then the FMAs (fewer serial steps per block)
#pragma unroll
      for (int j0 = 0; j0 < kUmChunkBlocks; j0 += JB) {
        uint32_t r[JB][CW];
#pragma unroll
        for (int jb = 0; jb < JB; ++jb) {
          const int g = 4 * cl + j0 + jb, t = g % G::NBUF, vv = g / G::NBUF;
          if (!um_wait_warp(&accfull[t], (uint32_t)(vv & 1), abort, p.status)) { ok = false; break; }
          tc05_fence_after();
          const uint32_t ta = tmem + lq + (uint32_t)(t * G::NACC + u * CW);
          if constexpr (CW == 8) tmem_ld8(ta, r[jb]);  // one sum per input (x_hi + x_lo)
          else tmem_ld16(ta, r[jb]);
        }
        if (!ok) break;
#pragma unroll
        for (int jb = 0; jb < JB; ++jb) tmem_wait_ld<CW>(r[jb]);
        tc05_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int jb = 0; jb < JB; ++jb) mbar_arrive(&accempty[(4 * cl + j0 + jb) % G::NBUF]);
        }
#pragma unroll
        for (int jb = 0; jb < JB; ++jb) {
#pragma unroll
          for (int i = 0; i < CW; ++i) acc[i] = fmaf(dsc[j0 + jb], __uint_as_float(r[jb][i]), acc[i]);
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[s]);
    }

    // store: row of this thread and its CW inputs
    float accs[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) accs[i] = acc[i];
    const bool up = DUAL && v >= HR;
    const size_t row = rb + (size_t)(DUAL ? v % HR : v);
    if (p.S > 1 || !DUAL) {
      if (ok && row < p.rows) {
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int b = u * CW + i;
          if (b >= p.B) break;
          if (p.S > 1) {
            p.part[(((size_t)slice * (DUAL ? 2 : 1) + (up ? 1 : 0)) * p.B + b) * p.rows + row] = accs[i];
          } else {
            float yv = accs[i];
            if (p.bias) yv += p.bias[row];
            if (p.residual) yv = p.residual[(size_t)b * p.y_stride + row] + yv;
            p.y[(size_t)b * p.y_stride + row] = yv;
          }
        }
      }
    } else {
      // dual, one slice: the up rows hand their sums to the gate rows
      // through shared memory (the ring, once the epilogue warps are done;
      // every copy and MMA has completed by then)
      float* xch = reinterpret_cast<float*>(gbase);  // [NP][HR]
      named_barrier_sync(1, 32 * G::EPI);
      if (up) {
#pragma unroll
        for (int i = 0; i < CW; ++i) xch[(size_t)(u * CW + i) * HR + (v - HR)] = accs[i];
      }
      named_barrier_sync(1, 32 * G::EPI);
      if (!up && ok && row < p.rows) {
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int b = u * CW + i;
          if (b >= p.B) break;
          p.y[(size_t)b * p.y_stride + row] = silu(accs[i]) * xch[(size_t)b * HR + v];
        }
      }
    }
    tc05_fence_before();
  }

  pdl_launch_dependents();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc05_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(G::TMEM_COLS)
                 : "memory");
  }
}

// Sum of the S slices' partials in slice order, then the epilogue.
template <bool DUAL>
__global__ void __launch_bounds__(256) um_reduce_kernel(UmParams p) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int H2 = DUAL ? 2 : 1;
  const size_t n = (size_t)p.B * p.nrows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / p.nrows, row = p.row0 + (i - b * p.nrows);
    float v[H2];
#pragma unroll
    for (int hh = 0; hh < H2; ++hh) {
      v[hh] = 0.0f;
      for (int sl = 0; sl < p.S; ++sl) v[hh] += p.part[(((size_t)sl * H2 + hh) * p.B + b) * p.rows + row];
    }
    float y;
    if (DUAL) {
      y = silu(v[0]) * v[H2 - 1];
    } else {
      y = v[0];
      if (p.bias) y += p.bias[row];
      if (p.residual) y = p.residual[b * p.y_stride + row] + y;
    }
    p.y[b * p.y_stride + row] = y;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 um_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Raw weight rows: the row-major block stream as bytes [rows][row_bytes],
// boxes of one chunk (4 blocks) x box_rows rows, no swizzle.
minq_status um_weight_map(const void* w, size_t rows, int nb, int bb, int box_rows, CUtensorMap* out) {
  auto fn = um_encode_fn();
  if (!fn) return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const uint64_t row_bytes = (uint64_t)nb * bb;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(kUmChunkBlocks * bb), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (" + std::to_string((int)r) + ")");
  return MINQ_OK;
}

// Inputs x_hi / x_lo: bf16 [B][cols], boxes of 64 columns x N inputs with
// the 128-byte swizzle (rows past B read as zero).
minq_status um_input_map(const __nv_bfloat16* x, int B, int cols, int N, CUtensorMap* out) {
  auto fn = um_encode_fn();
  if (!fn) return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)N};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(x), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled (inputs) failed (" + std::to_string((int)r) + ")");
  return MINQ_OK;
}

template <int DT, int NP, bool DUAL>
minq_status um_launch(const void* w0, const void* w1, const __nv_bfloat16* xh,
                      const __nv_bfloat16* xl, int cols, UmParams p, unsigned tiles, cudaStream_t s) {
  using G = UmGeom<DT, NP>;
  constexpr int HR = DUAL ? G::ROWS / 2 : G::ROWS;
  CUtensorMap m0, m1, mh, ml;
  const int nb = cols / kBlock;
  MINQ_TRY(um_weight_map(w0, p.rows, nb, G::bb, HR, &m0));
  if (DUAL) {
    MINQ_TRY(um_weight_map(w1, p.rows, nb, G::bb, HR, &m1));
  } else {
    m1 = m0;
  }
  MINQ_TRY(um_input_map(xh, p.B, cols, NP, &mh));
  MINQ_TRY(um_input_map(xl, p.B, cols, NP, &ml));
  p.stages = std::min(G::max_stages(), std::max(2, p.slice_chunks));
  // at least 120 KB so one CTA holds an SM: its TMEM allocation never waits
  // for another CTA's
  const size_t smem = std::max<size_t>(G::smem(p.stages), 120 * 1024);
  auto k = qmm_umma_kernel<DT, NP, DUAL>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
  MINQ_CUDA_TRY(launch_k(k, dim3(tiles, (unsigned)p.S), dim3(G::THREADS), smem, s, m0, m1, mh, ml, p));
  if (p.S > 1) {
    const size_t n = (size_t)p.B * p.nrows;
    const unsigned gr = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    MINQ_CUDA_TRY(launch_k(um_reduce_kernel<DUAL>, dim3(gr), dim3(256), 0, s, p));
  }
  return MINQ_OK;
}

template <int DT, bool DUAL>
minq_status um_dispatch_n(const void* w0, const void* w1, const __nv_bfloat16* xh,
                          const __nv_bfloat16* xl, int cols, const UmParams& p, unsigned tiles,
                          cudaStream_t s) {
  if (p.B <= 16) return um_launch<DT, 16, DUAL>(w0, w1, xh, xl, cols, p, tiles, s);
  if (p.B <= 32) return um_launch<DT, 32, DUAL>(w0, w1, xh, xl, cols, p, tiles, s);
  return um_launch<DT, 64, DUAL>(w0, w1, xh, xl, cols, p, tiles, s);
}

}  // namespace

bool qmatmul_umma_takes(int dtype, int cols, int B, size_t xp_floats) {
  return (dtype == MINQ_Q4_0 || dtype == MINQ_Q8_0) && B >= 1 && B <= 64 && cols > 0 &&
         cols % (kUmChunkBlocks * kBlock) == 0 && xp_floats >= (size_t)B * cols;
}

minq_status launch_qmatmul_umma(int dtype, const void* w0, const void* w1, size_t rows, int cols,
                                int B, const float* x, size_t x_stride, const float* norm_w,
                                float eps, float* xp, size_t xp_floats, const float* bias,
                                const float* residual, float* y, size_t y_stride, float* part,
                                size_t part_floats, cudaStream_t s) {
  if (!qmatmul_umma_takes(dtype, cols, B, xp_floats) || rows == 0)
    return fail(MINQ_ERR_ARG, "tcgen05 batched matvec: dtype, shape or scratch");
  if ((uintptr_t)w0 % 16 || (w1 && (uintptr_t)w1 % 16) || (uintptr_t)xp % 16 ||
      (uintptr_t)x % 16 || x_stride % 4 || (norm_w && (uintptr_t)norm_w % 16))
    return fail(MINQ_ERR_ARG, "tcgen05 batched matvec operands must be 16-byte aligned");
  if (rows > (size_t)INT32_MAX) return fail(MINQ_ERR_SHAPE, "tcgen05 batched matvec: too many rows");
  __nv_bfloat16* xh = reinterpret_cast<__nv_bfloat16*>(xp);
  __nv_bfloat16* xl = xh + (size_t)B * cols;
  MINQ_CUDA_TRY(launch_k(um_xprep_kernel,
                         dim3((unsigned)B, (unsigned)((cols + kUmPrepCols - 1) / kUmPrepCols)),
                         dim3(128), 0, s, x, x_stride, cols, norm_w, eps,
                         dtype == MINQ_Q4_0 ? 1 : 0, xh, xl));
  UmParams p{};
  p.rows = rows;
  p.B = B;
  p.bias = bias;
  p.residual = residual;
  p.y = y;
  p.y_stride = y_stride;
  p.part = part;
  p.status = device_status_word();
  const bool dual = w1 != nullptr;
  const int rows_cta = 128;
  const int hr = dual ? rows_cta / 2 : rows_cta;
  const size_t tiles = (rows + hr - 1) / hr;
  p.nchunks = cols / (kUmChunkBlocks * kBlock);
  p.tile0 = 0;
  p.row0 = 0;
  p.nrows = rows;
  // K slices. Cost model in units of one full-K CTA's time: waves of CTAs
  // (one per SM) / slices, plus ~2 % per slice for the partials' reduce.
  // Single launch: S slices of every row tile. When the row tiles overrun
  // whole waves by a few (Qwen3-4B gate/up: 152 tiles on 148 SMs), the
  // overrun tiles go to a second launch split over the SMs instead of
  // taking a whole extra wave each.
  const size_t sms = (size_t)sm_count();
  const int halves = dual ? 2 : 1;
  const int smax = std::max(1, p.nchunks / 2);  // each slice at least two chunks
  auto fits = [&](int S) {
    return S == 1 || (part && (size_t)S * halves * B * rows <= part_floats);
  };
  constexpr double kRed = 0.02;
  double best = 1e30;
  int S = 1;
  for (int c = 1; c <= smax && fits(c); ++c) {
    const double cost = (double)((tiles * c + sms - 1) / sms) / c + (c > 1 ? kRed * c : 0.0);
    if (cost < best - 1e-9) {
      best = cost;
      S = c;
    }
  }
  static const bool plan_env = [] {  // MINQ_UM_PLAN=0: one wave-filling rule only
    const char* e = std::getenv("MINQ_UM_PLAN");
    return !(e && e[0] == '0');
  }();
  if (!plan_env) {
    S = (int)std::min<size_t>(std::max<size_t>(1, sms / tiles), (size_t)smax);
    while (S > 1 && !fits(S)) --S;
  }
  size_t head = tiles;
  int St = 1;
  if (plan_env && tiles > sms && tiles % sms != 0) {
    const size_t h = tiles / sms * sms, tail = tiles - h;
    int c = std::min(smax, (int)(sms / tail));
    while (c > 1 && !fits(c)) --c;
    const double cost = (double)(h / sms) + 1.0 / c + kRed * c * (double)tail / (double)tiles;
    if (c > 1 && cost < best - 1e-9) {
      head = h;
      St = c;
    }
  }
  auto go = [&](UmParams q, size_t t0, size_t nt, int slices) -> minq_status {
    q.tile0 = (int)t0;
    q.slice_chunks = (q.nchunks + slices - 1) / slices;
    q.S = (q.nchunks + q.slice_chunks - 1) / q.slice_chunks;
    q.row0 = t0 * hr;
    q.nrows = std::min(rows, (t0 + nt) * hr) - q.row0;
    if (dtype == MINQ_Q4_0)
      return dual ? um_dispatch_n<MINQ_Q4_0, true>(w0, w1, xh, xl, cols, q, (unsigned)nt, s)
                  : um_dispatch_n<MINQ_Q4_0, false>(w0, w1, xh, xl, cols, q, (unsigned)nt, s);
    return dual ? um_dispatch_n<MINQ_Q8_0, true>(w0, w1, xh, xl, cols, q, (unsigned)nt, s)
                : um_dispatch_n<MINQ_Q8_0, false>(w0, w1, xh, xl, cols, q, (unsigned)nt, s);
  };
  if (head < tiles) {
    MINQ_TRY(go(p, 0, head, 1));
    return go(p, head, tiles - head, St);
  }
  return go(p, 0, tiles, S);
}

}  // namespace minq
