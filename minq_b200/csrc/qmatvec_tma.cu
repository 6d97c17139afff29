// TMA-fed batch-1 quantized matvec (QuantizedTensor::matvec, quantize.rs:
// 215-280) for rows whose byte length is a multiple of 16 (cols % 128 == 0).
//
// The weight is described to the TMA unit as a 2-D tensor of 32-bit words
// [rows][row_bytes/4] in the reference's AoS block layout, so ONE
// cp.async.bulk.tensor.2d instruction fetches a box of nr rows x one chunk
// of CK blocks (Q4_0: 32 blocks = 640 B per row, Q8_0: 16 blocks = 576 B per
// row) into shared memory. Wide box rows keep every DRAM burst long.
//
// CTA = 8 consumer warps + 1 producer warp and owns nr consecutive output
// rows (nr <= 32, or 16 gate/up pairs) and every column; nr is chosen per
// launch so the grid is a whole number of waves over the SMs. Chunks stream
// through an S-deep ring (stage = one box, or two in the SwiGLU dual mode);
// every consumer warp reads every stage. Warp w owns rows w, w+8, ...; in a
// warp, lane = 4*block + sub covers 8 columns of one of 8 consecutive blocks
// and loops over the chunk's blocks in steps of 8, reusing its 8 x-values
// for all of the warp's rows. Each row is thus reduced inside one warp
// (shuffles, fixed order) and the epilogue (bias / residual / SwiGLU) writes
// y. The producer primes the ring before waiting on the previous kernel
// (PDL), so weight traffic overlaps the hand-over between kernels.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "kernels.h"
#include "ktimer.h"
#include "matvec_common.cuh"
#include "pipeline.cuh"

namespace minq {

constexpr int kCW = 8;      // consumer warps
constexpr int kMaxS = 16;   // max ring depth

template <int DT>
struct QmvGeom {
  static constexpr int BB = DT == MINQ_Q8_0 ? kQ8Bytes : kQ4Bytes;
  static constexpr int CK = DT == MINQ_Q8_0 ? 16 : 32;  // blocks per chunk
  static constexpr int CKB = CK * BB;                     // bytes per box row (576 / 640)
};

template <bool DUAL>
struct QmvLimits {
  static constexpr int NRMAX = DUAL ? 16 : 32;   // rows (pairs) per CTA
  static constexpr int RPW = NRMAX / kCW;        // rows (pairs) per warp
};

template <int DT, bool DUAL>
__global__ void __launch_bounds__(32 * (kCW + 1), 2)
    qmatvec_tma_kernel(const __grid_constant__ CUtensorMap tm0,
                       const __grid_constant__ CUtensorMap tm1, MatvecParams p, QmvPlan t) {
  using Gm = QmvGeom<DT>;
  constexpr int BB = Gm::BB, CK = Gm::CK, CKB = Gm::CKB;
  constexpr int RPW = QmvLimits<DUAL>::RPW;
  constexpr int NACC = DUAL ? 2 * RPW : RPW;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int S = t.stages, nr = t.nr;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kMaxS;
  uint64_t* xbar = empty + kMaxS;
  float* red = reinterpret_cast<float*>(smem_raw + 8 * (2 * kMaxS + 1) + 8);  // 33 floats
  float* xs = reinterpret_cast<float*>(smem_raw + 512);
  float* ws = xs + p.cols;
  unsigned char* ring = reinterpret_cast<unsigned char*>(ws + (p.norm_w ? p.cols : 0));
  const int box_bytes = nr * CKB;
  const int box_stride = (box_bytes + 127) & ~127;  // TMA destinations are 128-B aligned
  const int stage_bytes = (DUAL ? 2 : 1) * box_stride;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * nr;
  const int nb = p.cols / kBlock;
  const int nchunks = t.nchunks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    mbar_init(xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();

  int pc = 0;  // producer's next chunk
  auto produce = [&](int c) -> bool {
    const int s = c % S;
    if (!mbar_wait(&empty[s], ((uint32_t)(c / S) & 1u) ^ 1u, p.status)) return false;
    if (lane == 0) {
      unsigned char* dst = ring + (size_t)s * stage_bytes;
      mbar_arrive_expect_tx(&full[s], (uint32_t)((DUAL ? 2 : 1) * box_bytes));
      tma_load_2d_nohint(dst, &tm0, c * (CKB / 4), r0, &full[s]);
      if (DUAL) tma_load_2d_nohint(dst + box_stride, &tm1, c * (CKB / 4), r0, &full[s]);
    }
    __syncwarp();
    return true;
  };

  // Weights do not depend on the previous kernel: start streaming them first.
  if (warp == kCW) {
    for (; pc < S && pc < nchunks; ++pc) produce(pc);
  }
  pdl_wait();
  if (threadIdx.x == 0) {
    const uint32_t xb = (uint32_t)p.cols * 4u;
    mbar_arrive_expect_tx(xbar, p.norm_w ? 2u * xb : xb);
    bulk_g2s(xs, p.x, xb, xbar);
    if (p.norm_w) bulk_g2s(ws, p.norm_w, xb, xbar);
  }
  mbar_wait(xbar, 0u, p.status);  // a timeout sets the status word; carry on uniformly
  if (p.norm_w) block_rms_scale(p, xs, ws, red, true);
  else __syncthreads();
  pdl_launch_dependents();

  if (warp == kCW) {
    bool ok = true;
    for (; pc < nchunks && ok; ++pc) ok = produce(pc);
    for (int c = max(0, nchunks - S); ok && c < nchunks; ++c)  // drain
      ok = mbar_wait(&empty[c % S], (uint32_t)(c / S) & 1u, p.status);
    return;
  }

  // Consumers: warp owns local rows warp + 8*i (i < RPW).
  const int bi = lane >> 2, sub = lane & 3;
  float acc[NACC];
#pragma unroll
  for (int i = 0; i < NACC; ++i) acc[i] = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    const int s = c % S;
    if (!mbar_wait(&full[s], (uint32_t)(c / S) & 1u, p.status)) break;
    const unsigned char* box = ring + (size_t)s * stage_bytes;
#pragma unroll
    for (int j = 0; j < CK / 8; ++j) {
      const int bl = j * 8 + bi;
      const int bg = c * CK + bl;
      if (bg < nb) {
        const float4 xa = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub);
        const float4 xb = *reinterpret_cast<const float4*>(xs + 32 * bg + 8 * sub + 4);
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          const int rl = warp + kCW * i;
          if (rl < nr) {
            const unsigned char* blk = box + rl * CKB + bl * BB;
            acc[i] = fmaf(*reinterpret_cast<const float*>(blk),
                          lane_dot_smem<DT>(blk, sub, xa, xb), acc[i]);
            if (DUAL) {
              const unsigned char* blk1 = blk + box_stride;
              acc[RPW + i] = fmaf(*reinterpret_cast<const float*>(blk1),
                                  lane_dot_smem<DT>(blk1, sub, xa, xb), acc[RPW + i]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
#pragma unroll
  for (int i = 0; i < NACC; ++i) acc[i] = warp_sum(acc[i]);
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int rl = warp + kCW * i;
    const size_t r = (size_t)r0 + rl;
    if (lane == i && rl < nr && r < p.rows) {
      float v;
      if (DUAL) {
        v = silu(acc[i]) * acc[RPW + i];
      } else {
        v = acc[i];
        if (p.bias) v += p.bias[r];
        if (p.residual) v = p.residual[r] + v;
      }
      p.y[r] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side: plan + tensor-map encoding (driver entry point via the runtime).

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

static int chunk_bytes(int dtype) {
  return dtype == MINQ_Q8_0 ? QmvGeom<MINQ_Q8_0>::CKB : QmvGeom<MINQ_Q4_0>::CKB;
}

QmvPlan plan_qmatvec_tma(int dtype, bool dual, size_t rows, int cols, bool norm) {
  const int sms = sm_count();
  const int nrmax = dual ? QmvLimits<true>::NRMAX : QmvLimits<false>::NRMAX;
  const size_t slots = (size_t)sms * 2;  // two CTAs per SM
  QmvPlan t{};
  // Smallest k such that rows split over k full waves fit nrmax rows per CTA.
  size_t k = 1;
  while ((rows + k * slots - 1) / (k * slots) > (size_t)nrmax) ++k;
  t.nr = (int)std::max<size_t>(1, (rows + k * slots - 1) / (k * slots));
  t.nctas = (rows + t.nr - 1) / t.nr;
  const int ckb = chunk_bytes(dtype);
  const size_t row_bytes = (size_t)(cols / kBlock) * block_bytes(dtype);
  t.nchunks = (int)((row_bytes + ckb - 1) / ckb);
  const size_t box = ((size_t)t.nr * ckb + 127) & ~(size_t)127;
  const size_t stage = (dual ? 2 : 1) * box;
  const size_t fixed = 512 + (size_t)cols * 4 * (norm ? 2 : 1);
  // ring: ~40 KB of weight stages (at least 2), two CTAs per SM
  size_t S = std::max<size_t>(2, 40960 / stage);
  S = std::min<size_t>({S, (size_t)kMaxS, (size_t)std::max(t.nchunks, 1)});
  while (S > 2 && fixed + S * stage > 110 * 1024) --S;
  t.stages = (int)S;
  t.smem = fixed + S * stage;
  return t;
}

minq_status encode_qmatvec_map(const void* w, size_t rows, int cols, int dtype, int nr,
                               CUtensorMap* out) {
  auto fn = encode_fn();
  if (!fn) return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const uint64_t row_bytes = (uint64_t)(cols / kBlock) * block_bytes(dtype);
  cuuint64_t dims[2] = {row_bytes / 4, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(chunk_bytes(dtype) / 4), (cuuint32_t)nr};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MINQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MINQ_OK;
}

template <int DT, bool DUAL>
static minq_status launch_inst(const CUtensorMap& a, const CUtensorMap& b, const MatvecParams& p,
                               const QmvPlan& t, cudaStream_t s) {
  auto k = qmatvec_tma_kernel<DT, DUAL>;
  MINQ_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), t.smem));
  MINQ_CUDA_TRY(
      launch_k(k, dim3((unsigned)t.nctas), dim3(32 * (kCW + 1)), t.smem, s, a, b, p, t));
  MINQ_LAUNCH_CHECK("qmatvec_tma_kernel");
  return MINQ_OK;
}

// `m0` / `m1`: tensor maps encoded with this plan's nr (or null to encode here).
minq_status launch_qmatvec_tma(const MatvecParams& p, int dtype, const QmvPlan& t,
                               const CUtensorMap* m0, const CUtensorMap* m1, cudaStream_t s) {
  CUtensorMap a, b;
  const bool dual = p.w1 != nullptr;
  if (!m0) {
    MINQ_TRY(encode_qmatvec_map(p.w0, p.rows, p.cols, dtype, t.nr, &a));
    m0 = &a;
  }
  if (dual && !m1) {
    MINQ_TRY(encode_qmatvec_map(p.w1, p.rows, p.cols, dtype, t.nr, &b));
    m1 = &b;
  }
  if (!dual) m1 = m0;
  if (dtype == MINQ_Q8_0)
    return dual ? launch_inst<MINQ_Q8_0, true>(*m0, *m1, p, t, s)
                : launch_inst<MINQ_Q8_0, false>(*m0, *m1, p, t, s);
  return dual ? launch_inst<MINQ_Q4_0, true>(*m0, *m1, p, t, s)
              : launch_inst<MINQ_Q4_0, false>(*m0, *m1, p, t, s);
}

}  // namespace minq
