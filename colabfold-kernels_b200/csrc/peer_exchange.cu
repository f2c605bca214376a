// All-to-all over NVLink peer memory with the library's own kernels: plain 16-byte stores into the peers' receive
// buffers (no TMA, no multicast) and a flag barrier with bounded waits.  For the row-sharded Evoformer block, whose
// operands switch between row and column sharding (and, for the triangle multiplication, to channel shards and back)
// ten times per block: an NCCL all-to-all of 33-67 MB per rank reaches a third of the link rate there.
//
// The receive buffers and the flag array live in symmetric memory (same allocation on every rank, each rank holding
// the others' device pointers); nothing here allocates or synchronises the host.
#include "cfk_common.cuh"

namespace cfk {
namespace {

// Every rank tells every other that all it sent before this point has been written, then waits for the same from all.
// flags[r] is rank r's array of `parts` counters; counter[0] on this device numbers the barriers (it lives on the device
// so that a replayed CUDA graph counts on).  One thread per peer; called by one whole block.
__device__ void peer_barrier(int* const* __restrict__ flag_ptrs, int* __restrict__ counter, int rank, int parts, int* status,
                             int code) {
  __shared__ int s_epoch;
  if (threadIdx.x == 0) s_epoch = *counter + 1;
  __syncthreads();
  const int epoch = s_epoch;
  const int p = threadIdx.x;
  if (p < parts) {
    __threadfence_system();  // the data stores before this point are ordered before the flag
    int* theirs = flag_ptrs[p] + rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(theirs), "r"(epoch) : "memory");
    const int* mine = flag_ptrs[rank] + p;
    const long long t0 = clock64();
    bool ok = false;
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (v - epoch >= 0) { ok = true; break; }
      if (clock64() - t0 > (1ll << 31)) break;   // about a second: a peer is missing
    }
    if (!ok) report_timeout(status, code);
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = epoch;
}

__global__ void peer_barrier_kernel(int* const* __restrict__ flag_ptrs, int* __restrict__ counter, int rank, int parts,
                                    int* status, int code) {
  peer_barrier(flag_ptrs, counter, rank, parts, status, code);
}

// Part p of the send buffer goes to rank p.  A part is `rows` runs of `run16` 16-byte pieces: run i of part p starts
// src_part * p + src_row * i pieces into the send buffer and lands dst_part * rank + dst_row * i pieces into rank p's
// receive buffer, so that a switch between row and column sharding needs no packing copy before and no re-layout copy
// after the exchange (a plain [parts][chunk] all-to-all is rows = 1).
struct PeerCopy {
  int64_t rows, run16, src_part, src_row, dst_part, dst_row;
};

__global__ void __launch_bounds__(256) peer_alltoall_kernel(const uint4* __restrict__ send, void* const* __restrict__ recv_ptrs,
                                                            int rank, int parts, PeerCopy c, int blocks_per_part,
                                                            int* const* __restrict__ flag_ptrs, int* __restrict__ counter,
                                                            int* status, int code) {
  const int p = blockIdx.x / blocks_per_part, b = blockIdx.x % blocks_per_part;
  // start with the next rank so that the ranks do not all write to the same peer at the same time
  const int peer = (rank + 1 + p) % parts;
  const uint4* src = send + int64_t(peer) * c.src_part;
  uint4* dst = static_cast<uint4*>(recv_ptrs[peer]) + int64_t(rank) * c.dst_part;
  const int64_t total = c.rows * c.run16, stride = int64_t(blocks_per_part) * blockDim.x;
  auto so = [&](int64_t i) { const int64_t r = i / c.run16; return r * c.src_row + (i - r * c.run16); };
  auto dof = [&](int64_t i) { const int64_t r = i / c.run16; return r * c.dst_row + (i - r * c.run16); };
  int64_t i = int64_t(b) * blockDim.x + threadIdx.x;
  // four independent 16-byte transfers in flight per thread
  for (; i + 3 * stride < total; i += 4 * stride) {
    const uint4 v0 = src[so(i)], v1 = src[so(i + stride)], v2 = src[so(i + 2 * stride)], v3 = src[so(i + 3 * stride)];
    dst[dof(i)] = v0;
    dst[dof(i + stride)] = v1;
    dst[dof(i + 2 * stride)] = v2;
    dst[dof(i + 3 * stride)] = v3;
  }
  for (; i < total; i += stride) dst[dof(i)] = src[so(i)];
  // the block that finishes last runs the barrier (counter[1] counts the finished blocks): no second launch
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(counter + 1, 1);
    s_last = done == int(gridDim.x) - 1;
    if (s_last) counter[1] = 0;
  }
  __syncthreads();
  if (s_last) peer_barrier(flag_ptrs, counter, rank, parts, status, code);
}

}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_peer_alltoall(const void* send, const void* recv_ptrs, const void* flag_ptrs, void* counter, int rank,
                                 int parts, int64_t rows, int64_t run_bytes, int64_t src_part_bytes, int64_t src_row_bytes,
                                 int64_t dst_part_bytes, int64_t dst_row_bytes, void* stream) {
  if (!send || !recv_ptrs || !flag_ptrs || !counter) return CFK_ERR_NULL;
  if (parts < 1 || parts > 32 || rank < 0 || rank >= parts || rows < 0 || run_bytes < 0) return CFK_ERR_SHAPE;
  if ((run_bytes | src_part_bytes | src_row_bytes | dst_part_bytes | dst_row_bytes) % 16 != 0 || !aligned16(send)) return CFK_ERR_ALIGN;
  int* status = device_status_word();
  if (status == nullptr) return CFK_ERR_LAUNCH;
  auto st = static_cast<cudaStream_t>(stream);
  const PeerCopy c{rows, run_bytes / 16, src_part_bytes / 16, src_row_bytes / 16, dst_part_bytes / 16, dst_row_bytes / 16};
  const int64_t total = c.rows * c.run16;
  if (total > 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int bpp = (2 * sms + parts - 1) / parts;   // about two blocks per SM in all
    if (int64_t(bpp) * 256 > total) bpp = int((total + 255) / 256);
    if (bpp < 1) bpp = 1;
    peer_alltoall_kernel<<<bpp * parts, 256, 0, st>>>(static_cast<const uint4*>(send), static_cast<void* const*>(recv_ptrs), rank,
                                                      parts, c, bpp, static_cast<int* const*>(flag_ptrs),
                                                      static_cast<int*>(counter), status, 1901);
    return check_launch();
  }
  peer_barrier_kernel<<<1, 32, 0, st>>>(static_cast<int* const*>(flag_ptrs), static_cast<int*>(counter), rank, parts, status, 1901);
  return check_launch();
}
