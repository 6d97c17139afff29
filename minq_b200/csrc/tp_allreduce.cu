// One-shot all-reduce of the residual stream over the tensor-parallel ranks
// through NVLink peer memory: the collective after o_proj and after
// down_proj of every layer (model.rs:304, :313 with the rows / columns of the
// projections split over the ranks), which sums hidden_size floats.
//
// Every rank owns a receive buffer [site][rank][hidden] and per-CTA flags
// [site][rank][cta] (one site per all-reduce of a token: 2 per layer), mapped
// into every other rank by CUDA IPC at minq_tp_init. CTA c of the kernel
//   1. stores its slice of x into slot [site][this rank] of every rank's
//      buffer (peer stores over NVLink; its own buffer locally),
//   2. after a system-scope fence, writes the epoch into flag
//      [site][this rank][c] of every rank,
//   3. waits (bounded: 1 s of %globaltimer, then the device status word is
//      set and x is left unsummed) until flag [site][q][c] of its own buffer
//      holds the epoch for every rank q,
//   4. writes x[slice] = sum over q = 0, 1, ... of the slots, in rank order,
//      so every rank ends with the same bits.
// The epoch is a per-model token counter in device memory, advanced once per
// token after its last all-reduce, so the kernels replay unchanged inside a
// captured CUDA graph. A site's slot is rewritten one token later only after
// every rank has finished that site (each rank's next write to it follows
// its own completion of every earlier site, which needed all ranks' data).
// No load of peer memory is made here (the peers push), and nothing uses
// cluster multicast.
#include <unistd.h>

#include <cstring>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "nccl_dl.h"
#include "pipeline.cuh"

namespace minq {

namespace {

constexpr int kArThreads = 128;
constexpr int kArCols = 4 * kArThreads;  // floats per CTA

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads) tp_ar_kernel(float* __restrict__ x, int H, int world,
                                                          int rank, int site,
                                                          const unsigned long long* step,
                                                          float* const* peer_recv,
                                                          int* const* peer_flag,
                                                          const float* recv, const int* flag,
                                                          int* status) {
  pdl_wait();
  __shared__ int ok;
  const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
  const int c = cta * kArCols + 4 * tid;
  const bool act = c < H;
  const int ep = (int)(*step + 1ull);
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (act) v = __ldcg(reinterpret_cast<const float4*>(x + c));
  const size_t slot = ((size_t)site * world + rank) * H;
  for (int p = 0; p < world; ++p)
    if (act) __stcg(reinterpret_cast<float4*>(peer_recv[p] + slot + c), v);
  if (tid == 0) ok = 1;
  __syncthreads();
  if (tid < world) {
    __threadfence_system();  // this CTA's slice is visible to every rank before its flag
    st_release_sys(peer_flag[tid] + ((size_t)site * world + rank) * ncta + cta, ep);
    const int* f = flag + ((size_t)site * world + tid) * ncta + cta;
    if (ld_acquire_sys(f) != ep) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(f) != ep) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(status, kDeviceTimeout);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  if (!ok || !act) return;
  const float* r = recv + (size_t)site * world * H + c;
  float4 s = __ldcg(reinterpret_cast<const float4*>(r));
  for (int q = 1; q < world; ++q) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(r + (size_t)q * H));
    s.x += t.x;
    s.y += t.y;
    s.z += t.z;
    s.w += t.w;
  }
  *reinterpret_cast<float4*>(x + c) = s;
}

__global__ void tp_ar_advance_kernel(unsigned long long* step) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) *step += 1ull;
}

struct ArPeerInfo {
  cudaIpcMemHandle_t handle;
  long long pid;
  unsigned long long ptr;
  int device;
  int ok;
};

}  // namespace

bool tp_ar_wanted() {
  const char* e = getenv("MINQ_TP_NCCL");
  return !(e && e[0] == '1');
}

minq_status tp_ar_setup(TpAr* ar, int rank, int world, int H, int sites, void* nccl_comm,
                        cudaStream_t s) {
  *ar = TpAr{};
  if (world < 2 || H % 4 != 0) return MINQ_OK;  // the NCCL path serves these
  const NcclApi& nc = nccl_api();
  const int ncta = (H + kArCols - 1) / kArCols;
  // 8 bytes per element: the per-op kernel's f32 slots use the first half,
  // the decode megakernel's (value, epoch) pairs all of it
  const size_t recv_bytes = (size_t)sites * world * H * 8;
  const size_t flag_bytes = (size_t)sites * world * ncta * 4;
  const size_t recv_pad = (recv_bytes + 255) & ~(size_t)255;
  const size_t ctr_off = (recv_pad + flag_bytes + 255) & ~(size_t)255;
  const size_t bytes = ctr_off + 256;  // + the decode megakernel's exchange epoch
  int dev = 0;
  MINQ_CUDA_TRY(cudaGetDevice(&dev));
  char* buf = nullptr;
  MINQ_CUDA_TRY(cudaMalloc(&buf, bytes));
  MINQ_CUDA_TRY(cudaMemset(buf, 0, bytes));
  MINQ_CUDA_TRY(cudaDeviceSynchronize());
  ar->base = buf;
  ar->recv = reinterpret_cast<float*>(buf);
  ar->flag = reinterpret_cast<int*>(buf + recv_pad);
  ar->ctr = reinterpret_cast<unsigned long long*>(buf + ctr_off);
  // exchange (IPC handle, pid, pointer, device) with every rank: each rank
  // fills its own row, a byte-sum all-reduce gathers them
  ArPeerInfo mine{};
  mine.ok = cudaIpcGetMemHandle(&mine.handle, buf) == cudaSuccess ? 1 : 0;
  mine.pid = (long long)getpid();
  mine.ptr = (unsigned long long)(uintptr_t)buf;
  mine.device = dev;
  std::vector<ArPeerInfo> all(world);
  std::memset(all.data(), 0, sizeof(ArPeerInfo) * world);
  all[rank] = mine;
  unsigned char* d_info = nullptr;
  MINQ_CUDA_TRY(cudaMalloc(&d_info, sizeof(ArPeerInfo) * world));
  MINQ_CUDA_TRY(cudaMemcpy(d_info, all.data(), sizeof(ArPeerInfo) * world, cudaMemcpyHostToDevice));
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
  ncclResult_t r = nc.AllReduce(d_info, d_info, sizeof(ArPeerInfo) * world, ncclUint8, ncclSum,
                                static_cast<ncclComm_t>(nccl_comm), s);
  r = nccl_settle(static_cast<ncclComm_t>(nccl_comm), r, deadline);
  cudaError_t e = cudaStreamSynchronize(s);
  if (r == ncclSuccess && e == cudaSuccess)
    e = cudaMemcpy(all.data(), d_info, sizeof(ArPeerInfo) * world, cudaMemcpyDeviceToHost);
  cudaFree(d_info);
  if (r != ncclSuccess) return fail(MINQ_ERR_NCCL, std::string("ncclAllReduce: ") + nc.GetErrorString(r));
  MINQ_CUDA_TRY(e);
  // map every peer's buffer: another process through its IPC handle, this
  // process's own allocation (a rank per thread) directly with peer access
  std::vector<float*> precv(world);
  std::vector<int*> pflag(world);
  int ok = 1;
  for (int q = 0; q < world && ok; ++q) {
    char* pb = nullptr;
    if (q == rank) {
      pb = buf;
    } else if (!all[q].ok) {
      ok = 0;
    } else if (all[q].pid == mine.pid) {
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, dev, all[q].device) != cudaSuccess || !can) {
        ok = 0;
      } else {
        const cudaError_t pe = cudaDeviceEnablePeerAccess(all[q].device, 0);
        if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) ok = 0;
        cudaGetLastError();
        pb = reinterpret_cast<char*>((uintptr_t)all[q].ptr);
      }
    } else {
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[q].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess) {
        pb = static_cast<char*>(p);
        ar->opened.push_back(p);
      } else {
        cudaGetLastError();
        ok = 0;
      }
    }
    if (pb) {
      precv[q] = reinterpret_cast<float*>(pb);
      pflag[q] = reinterpret_cast<int*>(pb + recv_pad);
    }
  }
  // every rank takes the peer path or none does
  int* d_ok = nullptr;
  MINQ_CUDA_TRY(cudaMalloc(&d_ok, sizeof(int)));
  MINQ_CUDA_TRY(cudaMemcpy(d_ok, &ok, sizeof(int), cudaMemcpyHostToDevice));
  r = nc.AllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(nccl_comm), s);
  r = nccl_settle(static_cast<ncclComm_t>(nccl_comm), r, deadline);
  e = cudaStreamSynchronize(s);
  if (r == ncclSuccess && e == cudaSuccess) e = cudaMemcpy(&ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d_ok);
  if (r != ncclSuccess) return fail(MINQ_ERR_NCCL, std::string("ncclAllReduce: ") + nc.GetErrorString(r));
  MINQ_CUDA_TRY(e);
  if (!ok) {
    tp_ar_release(ar);
    return MINQ_OK;  // the NCCL all-reduce stays in use
  }
  MINQ_CUDA_TRY(cudaMalloc(&ar->peer_recv, sizeof(float*) * world));
  MINQ_CUDA_TRY(cudaMalloc(&ar->peer_flag, sizeof(int*) * world));
  MINQ_CUDA_TRY(cudaMalloc(&ar->step, sizeof(unsigned long long)));
  MINQ_CUDA_TRY(cudaMemset(ar->step, 0, sizeof(unsigned long long)));
  MINQ_CUDA_TRY(cudaMemcpy(ar->peer_recv, precv.data(), sizeof(float*) * world, cudaMemcpyHostToDevice));
  MINQ_CUDA_TRY(cudaMemcpy(ar->peer_flag, pflag.data(), sizeof(int*) * world, cudaMemcpyHostToDevice));
  ar->world = world;
  ar->rank = rank;
  ar->sites = sites;
  ar->H = H;
  ar->ncta = ncta;
  ar->on = true;
  return MINQ_OK;
}

void tp_ar_release(TpAr* ar) {
  for (void* p : ar->opened) cudaIpcCloseMemHandle(p);
  ar->opened.clear();
  if (ar->base) cudaFree(ar->base);
  if (ar->peer_recv) cudaFree(ar->peer_recv);
  if (ar->peer_flag) cudaFree(ar->peer_flag);
  if (ar->step) cudaFree(ar->step);
  *ar = TpAr{};
}

minq_status launch_tp_allreduce(const TpAr& ar, float* x, int site, cudaStream_t s) {
  if (!ar.on || site < 0 || site >= ar.sites) return fail(MINQ_ERR_ARG, "peer all-reduce not set up");
  MINQ_CUDA_TRY(launch_k(tp_ar_kernel, dim3((unsigned)ar.ncta), dim3(kArThreads), 0, s, x, ar.H,
                         ar.world, ar.rank, site, (const unsigned long long*)ar.step,
                         (float* const*)ar.peer_recv, (int* const*)ar.peer_flag,
                         (const float*)ar.recv, (const int*)ar.flag, device_status_word()));
  return MINQ_OK;
}

minq_status launch_tp_ar_advance(const TpAr& ar, cudaStream_t s) {
  MINQ_CUDA_TRY(launch_k(tp_ar_advance_kernel, dim3(1), dim3(32), 0, s, ar.step));
  return MINQ_OK;
}

}  // namespace minq
