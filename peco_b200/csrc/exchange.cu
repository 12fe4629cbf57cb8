// Sequence <-> head reshard of the long-video configuration over NVLink peer
// memory (peco_b200/distributed.py drives it).
//
// Every rank owns a receive buffer and a flag array in memory that all ranks
// of the group have mapped (torch symmetric memory).  An exchange is one
// launch per rank of ``exchange_put_kernel``: its pieces -- equal-sized,
// contiguous row blocks -- are copied with 16-byte loads from local memory
// and 16-byte stores into the destination rank's buffer through its peer
// mapping (plain stores over NVLink; no TMA, no multicast).  The last block
// to finish raises this rank's flag in every destination's flag array to the
// exchange's epoch.  A receiver's ``exchange_wait_kernel`` then waits, with a
// bound, until every sender's flag has reached the epoch; kernels that follow
// it on the stream read the received data.
//
// Ordering: each block fences its stores at system scope before it counts
// itself done; the block that completes the count fences again and writes the
// flags with system-scope release stores; the waiter reads them with
// system-scope acquire loads.  An expired wait records kDevTimeout in the
// device status word and returns (the receive buffer is then incomplete and
// the call reports the error).
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

constexpr int kPutThreads = 256;

__device__ __forceinline__ void store_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ long long load_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct PutArgs {
  const unsigned char* src;
  const long long* src_off;           // [pieces] byte offsets in src
  const int* dst_rank;                // [pieces]
  const long long* dst_off;           // [pieces] byte offsets in the destination's buffer
  const unsigned long long* buffers;  // [world] every rank's receive buffer, as mapped here
  const unsigned long long* flags;    // [world] every rank's flag array, as mapped here
  long long piece_vecs;               // 16-byte vectors per piece
  int pieces, rank, world, flag_slot;
  long long epoch;
  unsigned* done;                     // blocks finished in this launch (reset by the last)
};

// grid (x: blocks per piece, y: pieces)
__global__ void __launch_bounds__(kPutThreads) exchange_put_kernel(const PutArgs a) {
  const int p = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(a.src + a.src_off[p]);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(a.buffers[a.dst_rank[p]]) + a.dst_off[p]);
  const long long stride = static_cast<long long>(gridDim.x) * kPutThreads;
  long long i = static_cast<long long>(blockIdx.x) * kPutThreads + threadIdx.x;
  // four vectors in flight per thread
  for (; i + 3 * stride < a.piece_vecs; i += 4 * stride) {
    const uint4 v0 = src[i], v1 = src[i + stride], v2 = src[i + 2 * stride], v3 = src[i + 3 * stride];
    dst[i] = v0;
    dst[i + stride] = v1;
    dst[i + 2 * stride] = v2;
    dst[i + 3 * stride] = v3;
  }
  for (; i < a.piece_vecs; i += stride) dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    if (atomicAdd(a.done, 1u) == total - 1) {
      __threadfence_system();
      // this rank's slot in every rank's flag array
      for (int q = 0; q < a.world; ++q) {
        long long* f = reinterpret_cast<long long*>(a.flags[q]) + static_cast<long long>(a.flag_slot) * a.world + a.rank;
        store_release_sys(f, a.epoch);
      }
      *a.done = 0u;  // ready for the next launch on this stream
    }
  }
}

// One thread per sender: bounded wait until its flag in this rank's array
// reaches ``epoch``.
__global__ void exchange_wait_kernel(const long long* flags, int world, int flag_slot, long long epoch,
                                     unsigned* status) {
  const int q = threadIdx.x;
  if (q >= world) return;
  const long long* f = flags + static_cast<long long>(flag_slot) * world + q;
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (load_acquire_sys(f) >= epoch) return;
    if ((it & 255u) == 255u && (globaltimer() - t0 > kWaitTimeoutNs || it > kWaitMaxSpins)) {
      record_status(status, kDevTimeout);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace
}  // namespace peco

using namespace peco;

extern "C" int peco_exchange_put(const void* src, const long long* src_offsets, const int* dst_ranks,
                                 const long long* dst_offsets, long long piece_bytes, int pieces,
                                 const unsigned long long* buffers, const unsigned long long* flags, int flag_slot,
                                 int rank, int world, long long epoch, unsigned* done_counter, void* stream) {
  if (!src || !src_offsets || !dst_ranks || !dst_offsets || !buffers || !flags || !done_counter) return kErrInvalidValue;
  if (pieces < 1 || pieces > 65535 || world < 1 || rank < 0 || rank >= world || flag_slot < 0 || epoch < 1)
    return kErrInvalidValue;
  if (piece_bytes < 16 || piece_bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16) return kErrInvalidValue;
  PutArgs a{static_cast<const unsigned char*>(src), src_offsets, dst_ranks, dst_offsets, buffers, flags,
            piece_bytes / 16, pieces, rank, world, flag_slot, epoch, done_counter};
  // about four blocks per SM over all pieces, at least one per piece
  long long per = (4LL * kNumSMs + pieces - 1) / pieces;
  const long long cap = (a.piece_vecs + kPutThreads - 1) / kPutThreads;
  per = per < cap ? per : cap;
  per = per < 1 ? 1 : per;
  exchange_put_kernel<<<dim3(static_cast<unsigned>(per), static_cast<unsigned>(pieces)), kPutThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

extern "C" int peco_exchange_wait(const long long* flags, int world, int flag_slot, long long epoch, void* stream) {
  if (!flags || world < 1 || world > 1024 || flag_slot < 0 || epoch < 1) return kErrInvalidValue;
  exchange_wait_kernel<<<1, 32 * ((world + 31) / 32), 0, static_cast<cudaStream_t>(stream)>>>(flags, world, flag_slot,
                                                                                             epoch, device_status_ptr());
  return launch_status();
}
