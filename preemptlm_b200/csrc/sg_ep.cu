// Expert-parallel token exchange over NVLink peer memory (row e): the
// dispatch and combine all-to-alls of one slotted MoE layer split over R
// GPUs, one process per GPU, without any host round trip.
//
// Every rank owns one region of device memory (cudaMalloc'd here, mapped into
// the other ranks' address spaces by CUDA IPC), laid out identically on all
// ranks (EpLayout):
//   rows  [R][CAP][H] bf16  token rows sent to this rank, one inbox per source
//   eid   [R][CAP]    int32 their local expert ids (-1: empty entry)
//   pid   [R][CAP]    int32 their pair ids at the source (t * k + j)
//   cnt   [R]         int32 rows in each inbox
//   ybuf  [CAP][H]    bf16  expert outputs of this rank's own pairs, in pair
//                           order, written back by the owning ranks
//   flag_in [R], flag_back [R] uint32: the step number whose inbox rows /
//                           outputs from rank s are complete
//   step              uint32 this rank's step counter (bumped by sg_ep_send;
//                           every later call of the step reads it, so a
//                           captured CUDA graph of the step replays correctly)
//   done [2]          uint32 finished-CTA counters of this rank's sg_ep_send
//                           and sg_ep_send_back (the last CTA publishes); one
//                           pair per region, so exchanges of different layers
//                           or groups never share a counter
// CAP = max tokens per step x k, the most pairs one source can route to one
// destination, so no inbox can overflow whatever the routing.
//
// A step (seq = 1, 2, ... in lockstep on all ranks, kept on the device):
//   sg_ep_send:      copy each pair's token row, expert id and pair id into
//                    the destination's inbox, at a position taken from a
//                    per-destination counter (the order within an inbox does
//                    not matter: outputs go back by pair id); the last CTA
//                    bumps the step number, publishes the counts, resets the
//                    counters and raises flag_in[me] = seq at every
//                    destination (system-scope release)
//   sg_ep_wait_inbox: acquire flag_in[s] >= seq for every source s, then mark
//                    the unused inbox entries empty (eid -1, ignored by
//                    sg_dispatch)
//   (sg_dispatch + sg_glu_forward run on the inboxes in place)
//   sg_ep_send_back: copy each output row to its source's ybuf at its pair
//                    id; the last CTA raises flag_back[me] = seq there
//   sg_ep_wait_back: acquire flag_back[d] >= seq for every destination d
//                    (on expiry the ybuf rows of the pairs sent to d are
//                    zeroed, so no earlier step's output is read as this one's)
//   (sg_combine reads ybuf)
// Buffer reuse across steps is safe by program order: a rank writes the next
// step's rows into a peer's inbox only after it saw that peer's outputs of
// this step (so the peer's GLU is done with its inbox), and writes outputs
// into a source's ybuf only after the source's next-step rows arrived (so
// the source's combine of the previous step is done).
//
// Every wait is bounded (two seconds of the global timer by default,
// sg_ep_set_wait_limit changes it per device); on expiry the kernel records
// SG_ERR_TIMEOUT (read with sg_device_status), empties the inbox or zeroes the
// output rows it was waiting for and returns.  After a timeout the exchange
// is out of step (a late peer may still write into this rank's region): the
// caller tears it down.  No TMA, no multicast: plain 16-byte peer loads and
// stores.
//
// Memory ordering of a hand-over (PTX memory model): every thread's row
// stores precede the CTA barrier; thread 0's fence.acq_rel.gpu (the
// __threadfence) then orders them before its atomicAdd on the done counter,
// so the CTA whose add returns gridDim.x - 1 observes, through that counter's
// release sequence, every CTA's rows (causality order is transitive at GPU
// scope).  Its fence.acq_rel.sys is cumulative: everything in its causal past,
// the other CTAs' peer stores included, is ordered before its following
// relaxed system-scope flag stores.  The receiver's ld.acquire.sys that reads
// the flag value synchronises with that fence, so the rows are visible to
// every later operation of the receiving thread, and the CTA barrier (or the
// kernel boundary) after it passes them on to the rest of the receiver.
#include <cuda_runtime.h>

#include <cstring>

#include "sg_common.cuh"

namespace sg {

__device__ int g_ep_status = 0;
// wait limit of the exchange kernels on this device, in global-timer nanoseconds
__device__ unsigned long long g_ep_wait_ns = 2000000000ull;

constexpr int EP_MAX_RANKS = 8;
constexpr long long EP_MAX_WAIT_US = 600LL * 1000 * 1000;  // upper bound of sg_ep_set_wait_limit

struct EpLayout {
  size_t rows, eid, pid, cnt, ybuf, flag_in, flag_back, step, done, bytes;
};

static size_t ep_align(size_t v) { return (v + 255) & ~size_t(255); }

static EpLayout ep_layout(int R, int cap, int H) {
  EpLayout l;
  size_t o = 0;
  l.rows = o;
  o += ep_align((size_t)R * cap * H * 2);
  l.eid = o;
  o += ep_align((size_t)R * cap * 4);
  l.pid = o;
  o += ep_align((size_t)R * cap * 4);
  l.cnt = o;
  o += ep_align((size_t)R * 4);
  l.ybuf = o;
  o += ep_align((size_t)cap * H * 2);
  l.flag_in = o;
  o += ep_align((size_t)R * 4);
  l.flag_back = o;
  o += ep_align((size_t)R * 4);
  l.step = o;
  o += 256;
  l.done = o;
  o += 256;
  l.bytes = o;
  return l;
}

struct EpPeers {
  uint8_t* base[EP_MAX_RANKS];  // every rank's region in this process's address space (own one included)
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for *flag >= seq (flags only grow); false on expiry.
__device__ bool ep_wait_flag(const uint32_t* flag, uint32_t seq) {
  if (ld_acquire_sys(flag) >= seq) return true;
  const unsigned long long t0 = global_ns(), limit = g_ep_wait_ns;
  while (true) {
    __nanosleep(256);
    if (ld_acquire_sys(flag) >= seq) return true;
    if (global_ns() - t0 > limit) {
      atomicCAS(&g_ep_status, 0, SG_ERR_TIMEOUT);
      return false;
    }
  }
}

// One row by one warp, 16-byte chunks, eight loads in flight per lane before
// their stores (a 4 KB row in one round trip; the destination is usually
// another GPU's memory).
__device__ __forceinline__ void copy_row(uint4* dst, const uint4* src, int chunks, int lane) {
  for (int c0 = lane; c0 < chunks; c0 += 256) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (c0 + 32 * u < chunks) v[u] = ldg_nc_v4(src + c0 + 32 * u);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (c0 + 32 * u < chunks) dst[c0 + 32 * u] = v[u];
  }
}

// Release / acquire fences at system scope (lighter than the sequentially
// consistent __threadfence_system).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// One warp per pair: its token row (H bf16) to the destination's inbox, plus
// its local expert id and pair id, at a slot taken from dcnt[destination]
// (zero on entry).  The last CTA to finish bumps the step number, publishes
// the counts and the step flag at every destination and zeroes dcnt.
__global__ void __launch_bounds__(256)
ep_send_kernel(EpPeers peers, int me, int R, int cap, int H, int k, int per, const uint16_t* __restrict__ x,
               const int32_t* __restrict__ inds, int32_t* __restrict__ dcnt, int P, size_t off_rows,
               size_t off_eid, size_t off_pid, size_t off_cnt, size_t off_flag_in, size_t off_step,
               size_t off_done) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int chunks = H >> 3;  // 16-byte chunks per row
  for (int p = gw; p < P; p += nw) {
    const int e = inds[p];  // the same for the whole warp
    if (e < 0 || e >= per * R) continue;
    const int d = e / per;
    int i = 0;
    if (lane == 0) i = atomicAdd(&dcnt[d], 1);
    i = __shfl_sync(0xffffffffu, i, 0);
    if (i >= cap) continue;  // cannot happen (at most P <= cap pairs per destination)
    uint8_t* dst_base = peers.base[d];
    const size_t slot = (size_t)me * cap + i;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(p / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(dst_base + off_rows + slot * H * 2);
    copy_row(dst, src, chunks, lane);
    if (lane == 0) {
      reinterpret_cast<int32_t*>(dst_base + off_eid)[slot] = e - d * per;
      reinterpret_cast<int32_t*>(dst_base + off_pid)[slot] = p;
    }
  }
  // The CTA barrier orders every thread's stores before thread 0's GPU-scope
  // fence and counter update; the last CTA's GPU-scope fence then has every
  // CTA's rows in its causal past, and its one system-scope fence (cumulative)
  // orders all of them before the flags.  A system fence costs microseconds,
  // so the kernel pays for exactly one.
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* done = reinterpret_cast<unsigned int*>(peers.base[me] + off_done);
    __threadfence();
    const unsigned prev = atomicAdd(&done[0], 1u);
    if (prev == gridDim.x - 1) {  // every CTA's rows are out: publish
      __threadfence();
      for (int d = 0; d < R; ++d)  // the count, and the counter back to zero for the next step
        reinterpret_cast<int32_t*>(peers.base[d] + off_cnt)[me] = atomicExch(&dcnt[d], 0);
      uint32_t* step = reinterpret_cast<uint32_t*>(peers.base[me] + off_step);
      const uint32_t seq = *step + 1;  // this step's number, read by the step's later kernels
      *step = seq;
      fence_acq_rel_sys();
      for (int d = 0; d < R; ++d) st_relaxed_sys(reinterpret_cast<uint32_t*>(peers.base[d] + off_flag_in) + me, seq);
      done[0] = 0;  // read again only by the next launch (kernel boundary)
    }
  }
}

// Block s: wait until source s's rows of step seq are in, then mark the rest
// of its inbox empty.  On expiry the whole inbox of s is marked empty.
__global__ void __launch_bounds__(256)
ep_wait_inbox_kernel(uint8_t* __restrict__ region, int cap, size_t off_eid, size_t off_cnt, size_t off_flag_in,
                     size_t off_step) {
  __shared__ int n;
  const int s = blockIdx.x;
  if (threadIdx.x == 0) {
    const uint32_t seq = *reinterpret_cast<const uint32_t*>(region + off_step);
    const bool ok = ep_wait_flag(reinterpret_cast<const uint32_t*>(region + off_flag_in) + s, seq);
    int c = ok ? reinterpret_cast<volatile int32_t*>(region + off_cnt)[s] : 0;
    n = (c < 0 || c > cap) ? 0 : c;
  }
  __syncthreads();
  int32_t* eid = reinterpret_cast<int32_t*>(region + off_eid) + (size_t)s * cap;
  for (int i = n + threadIdx.x; i < cap; i += blockDim.x) eid[i] = -1;
}

// One warp per inbox entry with a result: its output row back to the source's
// ybuf at the pair id.  The last CTA raises the step flag at every source.
__global__ void __launch_bounds__(256)
ep_send_back_kernel(EpPeers peers, int me, int R, int cap, int H, const uint8_t* __restrict__ region,
                    const uint16_t* __restrict__ y, size_t off_pid, size_t off_cnt, size_t off_ybuf,
                    size_t off_flag_back, size_t off_step, size_t off_done) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int chunks = H >> 3;
  const int32_t* cnt = reinterpret_cast<const int32_t*>(region + off_cnt);
  const int32_t* pid = reinterpret_cast<const int32_t*>(region + off_pid);
  for (int j = gw; j < R * cap; j += nw) {
    const int s = j / cap, i = j - s * cap;
    if (i >= cnt[s]) continue;
    const int p = pid[j];
    if (p < 0 || p >= cap) continue;
    const uint4* src = reinterpret_cast<const uint4*>(y + (size_t)j * H);
    uint4* dst = reinterpret_cast<uint4*>(peers.base[s] + off_ybuf + (size_t)p * H * 2);
    copy_row(dst, src, chunks, lane);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // as in ep_send_kernel: one system fence, by the last CTA
    unsigned int* done = reinterpret_cast<unsigned int*>(peers.base[me] + off_done);
    __threadfence();
    const unsigned prev = atomicAdd(&done[1], 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      fence_acq_rel_sys();
      const uint32_t seq = *reinterpret_cast<const uint32_t*>(region + off_step);
      for (int s = 0; s < R; ++s)
        st_relaxed_sys(reinterpret_cast<uint32_t*>(peers.base[s] + off_flag_back) + me, seq);
      done[1] = 0;
    }
  }
}

// Block d: wait until rank d's outputs of step seq are in ybuf.  On expiry
// the rows of this rank's pairs owned by d (inds[p] / per == d) are zeroed,
// one warp per row, so the combine never reads an earlier step's outputs.
__global__ void __launch_bounds__(256)
ep_wait_back_kernel(uint8_t* __restrict__ region, int H, const int32_t* __restrict__ inds, int P, int per,
                    size_t off_ybuf, size_t off_flag_back, size_t off_step) {
  __shared__ int ok;
  const int d = blockIdx.x;
  if (threadIdx.x == 0) {
    const uint32_t seq = *reinterpret_cast<const uint32_t*>(region + off_step);
    ok = ep_wait_flag(reinterpret_cast<const uint32_t*>(region + off_flag_back) + d, seq) ? 1 : 0;
  }
  __syncthreads();
  if (ok) return;
  const int lane = threadIdx.x & 31;
  const int chunks = H >> 3;
  for (int p = threadIdx.x >> 5; p < P; p += blockDim.x >> 5) {
    const int e = inds[p];
    if (e < 0 || e / per != d) continue;
    uint4* row = reinterpret_cast<uint4*>(region + off_ybuf + (size_t)p * H * 2);
    for (int c = lane; c < chunks; c += 32) row[c] = make_uint4(0, 0, 0, 0);
  }
}

int ep_device_status(int reset) {
  int v = 0;
  SG_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_ep_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SG_CUDA_TRY(cudaMemcpyToSymbol(g_ep_status, &zero, sizeof(int)));
  }
  return v;
}

static int ep_check(int R, int me, int cap, int H) {
  if (R < 1 || R > EP_MAX_RANKS || me < 0 || me >= R || cap < 1 || H < 8) return SG_ERR_INVALID_ARG;
  if (H % 8) return SG_ERR_SHAPE;
  return SG_OK;
}

// One warp per row while that fits 8 resident 256-thread CTAs per SM.
static int grid_for(int rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int want = (rows + 7) / 8;  // 8 warps per CTA, one row each
  return want < 1 ? 1 : (want < 8 * sms ? want : 8 * sms);
}

static EpPeers peers_of(void* const* bases, int R) {
  EpPeers p;
  for (int i = 0; i < EP_MAX_RANKS; ++i) p.base[i] = i < R ? static_cast<uint8_t*>(bases[i]) : nullptr;
  return p;
}

}  // namespace sg

// ============================================================== C-ABI
extern "C" long long sg_ep_region_bytes(int R, int cap, int H) {
  int st = sg::ep_check(R, 0, cap, H);
  if (st) return st;
  return (long long)sg::ep_layout(R, cap, H).bytes;
}

extern "C" int sg_ep_alloc(long long bytes, void** region) {
  if (bytes <= 0 || !region) return SG_ERR_INVALID_ARG;
  void* p = nullptr;
  SG_CUDA_TRY(cudaMalloc(&p, (size_t)bytes));
  const cudaError_t e = cudaMemset(p, 0, (size_t)bytes);  // flags start at step 0
  if (e != cudaSuccess) {
    cudaFree(p);
    return SG_ERR_CUDA;
  }
  SG_CUDA_TRY(cudaDeviceSynchronize());
  *region = p;
  return SG_OK;
}

extern "C" int sg_ep_free(void* region) {
  if (!region) return SG_OK;
  SG_CUDA_TRY(cudaFree(region));
  return SG_OK;
}

extern "C" int sg_ep_ipc_handle(void* region, uint8_t* handle64) {
  if (!region || !handle64) return SG_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  SG_CUDA_TRY(cudaIpcGetMemHandle(&h, region));
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return SG_OK;
}

extern "C" int sg_ep_ipc_open(const uint8_t* handle64, void** region) {
  if (!handle64 || !region) return SG_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  void* p = nullptr;
  SG_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *region = p;
  return SG_OK;
}

extern "C" int sg_ep_ipc_close(void* region) {
  if (!region) return SG_OK;
  SG_CUDA_TRY(cudaIpcCloseMemHandle(region));
  return SG_OK;
}

extern "C" int sg_ep_send(void* const* regions, int R, int me, int cap, int H, const uint16_t* x,
                          const int32_t* inds, int T, int k, int per, int32_t* dcnt, void* stream) {
  int st = sg::ep_check(R, me, cap, H);
  if (st) return st;
  if (T < 0 || k < 1 || per < 1) return SG_ERR_INVALID_ARG;
  const int P = T * k;
  if (P > cap) return SG_ERR_CAPACITY;
  if (!regions || (P > 0 && (!x || !inds)) || !dcnt) return SG_ERR_INVALID_ARG;
  for (int i = 0; i < R; ++i)
    if (!regions[i]) return SG_ERR_INVALID_ARG;
  const sg::EpLayout l = sg::ep_layout(R, cap, H);
  cudaStream_t s = (cudaStream_t)stream;
  sg::ep_send_kernel<<<sg::grid_for(P), 256, 0, s>>>(sg::peers_of(regions, R), me, R, cap, H, k, per, x, inds,
                                                       dcnt, P, l.rows, l.eid, l.pid, l.cnt, l.flag_in, l.step,
                                                       l.done);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_ep_wait_inbox(void* region, int R, int cap, int H, void* stream) {
  int st = sg::ep_check(R, 0, cap, H);
  if (st) return st;
  if (!region) return SG_ERR_INVALID_ARG;
  const sg::EpLayout l = sg::ep_layout(R, cap, H);
  sg::ep_wait_inbox_kernel<<<R, 256, 0, (cudaStream_t)stream>>>(static_cast<uint8_t*>(region), cap, l.eid, l.cnt,
                                                                 l.flag_in, l.step);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_ep_send_back(void* const* regions, int R, int me, int cap, int H, const uint16_t* y,
                               void* stream) {
  int st = sg::ep_check(R, me, cap, H);
  if (st) return st;
  if (!regions || !y) return SG_ERR_INVALID_ARG;
  for (int i = 0; i < R; ++i)
    if (!regions[i]) return SG_ERR_INVALID_ARG;
  const sg::EpLayout l = sg::ep_layout(R, cap, H);
  sg::ep_send_back_kernel<<<sg::grid_for(R * cap), 256, 0, (cudaStream_t)stream>>>(
      sg::peers_of(regions, R), me, R, cap, H, static_cast<const uint8_t*>(regions[me]), y, l.pid, l.cnt, l.ybuf,
      l.flag_back, l.step, l.done);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_ep_wait_back(void* region, int R, int cap, int H, const int32_t* inds, int T, int k, int per,
                               void* stream) {
  int st = sg::ep_check(R, 0, cap, H);
  if (st) return st;
  if (T < 0 || k < 1 || per < 1) return SG_ERR_INVALID_ARG;
  const long long P = (long long)T * k;
  if (P > cap) return SG_ERR_CAPACITY;
  if (!region || (P > 0 && !inds)) return SG_ERR_INVALID_ARG;
  const sg::EpLayout l = sg::ep_layout(R, cap, H);
  sg::ep_wait_back_kernel<<<R, 256, 0, (cudaStream_t)stream>>>(static_cast<uint8_t*>(region), H, inds, (int)P, per,
                                                                l.ybuf, l.flag_back, l.step);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_ep_set_wait_limit(long long microseconds) {
  if (microseconds < 1 || microseconds > sg::EP_MAX_WAIT_US) return SG_ERR_INVALID_ARG;
  const unsigned long long ns = (unsigned long long)microseconds * 1000ull;
  SG_CUDA_TRY(cudaMemcpyToSymbol(sg::g_ep_wait_ns, &ns, sizeof(ns)));
  return SG_OK;
}

// Byte offsets of the region's parts (rows, eid, pid, cnt, ybuf): the host
// wraps them as tensors for sg_dispatch / sg_glu_forward / sg_combine.
extern "C" int sg_ep_layout(int R, int cap, int H, long long* offsets5) {
  int st = sg::ep_check(R, 0, cap, H);
  if (st) return st;
  if (!offsets5) return SG_ERR_INVALID_ARG;
  const sg::EpLayout l = sg::ep_layout(R, cap, H);
  offsets5[0] = (long long)l.rows;
  offsets5[1] = (long long)l.eid;
  offsets5[2] = (long long)l.pid;
  offsets5[3] = (long long)l.cnt;
  offsets5[4] = (long long)l.ybuf;
  return SG_OK;
}
