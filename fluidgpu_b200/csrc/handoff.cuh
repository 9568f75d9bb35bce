// Hidden-state hand-off between the ranks of one NVLink node: the B200
// replacement of the reference's NCCL send/recv at task boundaries
// (executor.py:104-123, comm.py:24-46) and of the native runtime's
// IPC-buffer + flag and RDMA-write + flag handlers (comm_backend.cu:92-381,
// :1078-1187), whose device polling kernels spin without bound
// (comm_backend.cu:31-57).
//
// Mailbox (one allocation per rank, in that rank's HBM, mapped by every peer
// through CUDA IPC; all words 128-byte aligned):
//   data  [world][nslot][slot_bytes]   written by the sender (peer stores)
//   flags [world][nslot] u32           slot sequence number, sender-released
//   acks  [world][nslot] u32           acks of what THIS rank sent to each
//                                      peer, written remotely by the receiver
//   send_seq [world] u32, recv_seq [world] u32, tickets [2*world] u32 (local)
// Channel src -> dst uses dst's data[src][*] / flags[src][*] and src's
// acks[dst][*]. Message n of a channel goes to slot n % nslot.
//
// fg_handoff_put (on src): wait until acks[dst][slot] >= n - nslot (the
// receiver has drained the slot's previous message), store the payload into
// the peer slot with 16-byte stores, fence at system scope, and the last CTA
// (ticket) release-stores n into the peer flag.
// fg_handoff_recv (on dst): acquire-spin until flags[src][slot] >= n, copy
// the slot out, and the last CTA release-stores n into the sender's ack.
// Sequence numbers live on the device, so a captured CUDA graph can replay a
// put / recv any number of times. Every wait gives up after `timeout_ms`,
// records FG status 2 (peer flag timeout) and lets the kernel finish.
#pragma once
#include <cstring>

#include <cudaTypedefs.h>

#include "common.cuh"

namespace fg {
namespace handoff {

constexpr size_t kWordStride = 32;  // u32 words per flag / ack (128 bytes apart)

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// byte offsets of the regions for (world, nslot, slot_bytes)
struct Geometry {
  size_t data, flags, acks, send_seq, recv_seq, tickets, total;
  Geometry(int world, int nslot, size_t slot_bytes) {
    const size_t words = (size_t)world * nslot * kWordStride * 4;
    data = 0;
    flags = round_up((size_t)world * nslot * slot_bytes, 256);
    acks = flags + words;
    send_seq = acks + words;
    recv_seq = send_seq + (size_t)world * kWordStride * 4;
    tickets = recv_seq + (size_t)world * kWordStride * 4;
    total = tickets + (size_t)2 * world * kWordStride * 4;
  }
};

// grid-stride 16-byte copy, four loads in flight per thread before their
// stores (a remote store stream needs many outstanding requests)
__device__ __forceinline__ void copy16(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                       long long n16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 v0 = src[i], v1 = src[i + stride], v2 = src[i + 2 * stride], v3 = src[i + 3 * stride];
    dst[i] = v0;
    dst[i + stride] = v1;
    dst[i + 2 * stride] = v2;
    dst[i + 3 * stride] = v3;
  }
  for (; i < n16; i += stride) dst[i] = src[i];
}

struct PutArgs {
  const uint4* src;
  uint4* peer_slot0;        // peer data[me][0]
  uint32_t* peer_flags;     // peer flags[me][*]
  uint32_t* my_acks;        // my acks[dst][*]
  uint32_t* my_send_seq;    // my send_seq[dst]
  uint32_t* ticket;         // my tickets[dst]
  long long n16;            // payload in 16-byte units
  size_t slot_bytes;
  int nslot;
  uint64_t timeout_ns;
};

// Kernels that wait on another GPU let their dependents launch (PDL) only
// after the wait: a dependent launched earlier would sit in its own bounded
// pipeline waits for as long as the other GPU takes.
__global__ void __launch_bounds__(256) put_kernel(const PutArgs a) {
  griddep_wait();
  __shared__ uint32_t s_seq;
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const uint32_t seq = *((volatile uint32_t*)a.my_send_seq) + 1u;
    const int slot = (int)(seq % (uint32_t)a.nslot);
    // the receiver must have drained this slot's previous message
    if (seq > (uint32_t)a.nslot) wait_at_least(a.my_acks + slot * kWordStride, seq - a.nslot, a.timeout_ns, 0x401);
    s_seq = seq;
  }
  __syncthreads();
  griddep_launch_dependents();
  const uint32_t seq = s_seq;
  const int slot = (int)(seq % (uint32_t)a.nslot);
  copy16(a.peer_slot0 + (size_t)slot * (a.slot_bytes / 16), a.src, a.n16);
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(a.peer_flags + slot * kWordStride, seq);
    *a.ticket = 0u;
    *((volatile uint32_t*)a.my_send_seq) = seq;
  }
}

struct RecvArgs {
  uint4* out;
  const uint4* my_slot0;    // my data[src][0]
  const uint32_t* my_flags; // my flags[src][*]
  uint32_t* peer_acks;      // src's acks[me][*]
  uint32_t* my_recv_seq;    // my recv_seq[src]
  uint32_t* ticket;         // my tickets[world + src]
  long long n16;
  size_t slot_bytes;
  int nslot;
  uint64_t timeout_ns;
};

__global__ void __launch_bounds__(256) recv_kernel(const RecvArgs a) {
  griddep_wait();
  __shared__ uint32_t s_seq;
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const uint32_t seq = *((volatile uint32_t*)a.my_recv_seq) + 1u;
    wait_at_least(a.my_flags + (seq % (uint32_t)a.nslot) * kWordStride, seq, a.timeout_ns, 0x402);
    s_seq = seq;
  }
  __syncthreads();
  griddep_launch_dependents();
  const uint32_t seq = s_seq;
  const int slot = (int)(seq % (uint32_t)a.nslot);
  copy16(a.out, a.my_slot0 + (size_t)slot * (a.slot_bytes / 16), a.n16);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(a.peer_acks + slot * kWordStride, seq);  // slot may be reused
    *a.ticket = 0u;
    *((volatile uint32_t*)a.my_recv_seq) = seq;
  }
}

// Direct (zero-copy) hand-off on a one-slot mailbox: the producer's own
// kernel stores its output straight into the peer's slot (a peer pointer from
// fg_mailbox_slot), then signal_kernel publishes it; the consumer's
// wait_kernel spins until the flag arrives and later kernels read the slot in
// place. No slot acks: the channel is only used where the next message from
// the same sender depends on data the receiver produced after its last read
// of the slot (strict alternation between two ranks on the main path).
__global__ void signal_kernel(uint32_t* peer_flag, uint32_t* my_send_seq) {
  griddep_wait();  // the producer kernel's peer stores are complete
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t seq = *((volatile uint32_t*)my_send_seq) + 1u;
    *((volatile uint32_t*)my_send_seq) = seq;
    st_release_sys(peer_flag, seq);
  }
}

__global__ void wait_kernel(const uint32_t* my_flag, uint32_t* my_recv_seq, uint64_t timeout_ns) {
  griddep_wait();
  if (threadIdx.x == 0) {
    const uint32_t seq = *((volatile uint32_t*)my_recv_seq) + 1u;
    wait_at_least(my_flag, seq, timeout_ns, 0x403);
    *((volatile uint32_t*)my_recv_seq) = seq;
    __threadfence();
  }
  __syncwarp();
  griddep_launch_dependents();
}

// One CTA per 32 KiB, at most 128: small messages stay on a few SMs (only
// thread 0 of each CTA spins, so a waiting receive parks little on the SMs),
// large ones keep enough stores in flight to fill a peer link (~770 GB/s per
// direction).
inline int copy_grid(long long n16) {
  long long g = (n16 + 2047) / 2048;
  if (g > 128) g = 128;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace handoff
}  // namespace fg

extern "C" {

size_t fg_mailbox_bytes(int world, int nslot, size_t slot_bytes) {
  if (world <= 0 || nslot <= 0 || slot_bytes == 0 || slot_bytes % 16) return 0;
  return fg::handoff::Geometry(world, nslot, slot_bytes).total;
}

int fg_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
  FG_REQUIRE(ptr && handle_out && offset_out, "fg_ipc_export: null pointer");
  // IPC handles name whole allocations: find the one holding ptr
  static PFN_cuMemGetAddressRange_v3020 get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      fg::set_last_error("fg_ipc_export: cuMemGetAddressRange unavailable");
      return FG_ERR_CUDA;
    }
    get_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    fg::set_last_error("fg_ipc_export: pointer %p is not device memory", ptr);
    return FG_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    fg::set_last_error("fg_ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return FG_OK;
}

int fg_ipc_import(const void* handle, size_t offset, void** ptr_out) {
  FG_REQUIRE(handle && ptr_out, "fg_ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    fg::set_last_error("fg_ipc_import: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    (void)cudaGetLastError();
    return FG_ERR_PEER;
  }
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return FG_OK;
}

int fg_ipc_close(void* base_plus_offset, size_t offset) {
  FG_REQUIRE(base_plus_offset, "fg_ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(base_plus_offset) - offset);
  if (e != cudaSuccess) {
    fg::set_last_error("fg_ipc_close: %s", cudaGetErrorString(e));
    return FG_ERR_CUDA;
  }
  return FG_OK;
}

int fg_handoff_put(const void* src, size_t nbytes, void* my_mailbox, void* peer_mailbox, int world,
                   int me, int dst, int nslot, size_t slot_bytes, int timeout_ms, fg_stream_t stream) {
  using namespace fg::handoff;
  FG_REQUIRE(src && my_mailbox && peer_mailbox, "fg_handoff_put: null pointer");
  FG_REQUIRE(world > 0 && me >= 0 && me < world && dst >= 0 && dst < world && dst != me && nslot > 0,
             "fg_handoff_put: bad ranks me=%d dst=%d world=%d", me, dst, world);
  FG_REQUIRE(nbytes % 16 == 0 && nbytes <= slot_bytes && slot_bytes % 16 == 0,
             "fg_handoff_put: %zu bytes do not fit a %zu-byte slot (multiples of 16)", nbytes, slot_bytes);
  FG_REQUIRE(((uintptr_t)src & 15) == 0, "fg_handoff_put: src must be 16-byte aligned");
  const Geometry g(world, nslot, slot_bytes);
  uint8_t* mine = static_cast<uint8_t*>(my_mailbox);
  uint8_t* peer = static_cast<uint8_t*>(peer_mailbox);
  PutArgs a;
  a.src = static_cast<const uint4*>(src);
  a.peer_slot0 = reinterpret_cast<uint4*>(peer + g.data + (size_t)me * nslot * slot_bytes);
  a.peer_flags = reinterpret_cast<uint32_t*>(peer + g.flags) + (size_t)me * nslot * kWordStride;
  a.my_acks = reinterpret_cast<uint32_t*>(mine + g.acks) + (size_t)dst * nslot * kWordStride;
  a.my_send_seq = reinterpret_cast<uint32_t*>(mine + g.send_seq) + (size_t)dst * kWordStride;
  a.ticket = reinterpret_cast<uint32_t*>(mine + g.tickets) + (size_t)dst * kWordStride;
  a.n16 = (long long)(nbytes / 16);
  a.slot_bytes = slot_bytes;
  a.nslot = nslot;
  a.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
  return fg::launch_k("fg_handoff_put", put_kernel, dim3(copy_grid(a.n16)), dim3(256), 0,
                      (cudaStream_t)stream, a);
}

int fg_handoff_recv(void* out, size_t nbytes, void* my_mailbox, void* peer_mailbox, int world,
                    int me, int src, int nslot, size_t slot_bytes, int timeout_ms, fg_stream_t stream) {
  using namespace fg::handoff;
  FG_REQUIRE(out && my_mailbox && peer_mailbox, "fg_handoff_recv: null pointer");
  FG_REQUIRE(world > 0 && me >= 0 && me < world && src >= 0 && src < world && src != me && nslot > 0,
             "fg_handoff_recv: bad ranks me=%d src=%d world=%d", me, src, world);
  FG_REQUIRE(nbytes % 16 == 0 && nbytes <= slot_bytes && slot_bytes % 16 == 0,
             "fg_handoff_recv: %zu bytes do not fit a %zu-byte slot (multiples of 16)", nbytes, slot_bytes);
  FG_REQUIRE(((uintptr_t)out & 15) == 0, "fg_handoff_recv: out must be 16-byte aligned");
  const Geometry g(world, nslot, slot_bytes);
  uint8_t* mine = static_cast<uint8_t*>(my_mailbox);
  uint8_t* peer = static_cast<uint8_t*>(peer_mailbox);
  RecvArgs a;
  a.out = static_cast<uint4*>(out);
  a.my_slot0 = reinterpret_cast<const uint4*>(mine + g.data + (size_t)src * nslot * slot_bytes);
  a.my_flags = reinterpret_cast<const uint32_t*>(mine + g.flags) + (size_t)src * nslot * kWordStride;
  a.peer_acks = reinterpret_cast<uint32_t*>(peer + g.acks) + (size_t)me * nslot * kWordStride;
  a.my_recv_seq = reinterpret_cast<uint32_t*>(mine + g.recv_seq) + (size_t)src * kWordStride;
  a.ticket = reinterpret_cast<uint32_t*>(mine + g.tickets) + (size_t)(world + src) * kWordStride;
  a.n16 = (long long)(nbytes / 16);
  a.slot_bytes = slot_bytes;
  a.nslot = nslot;
  a.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
  return fg::launch_k("fg_handoff_recv", recv_kernel, dim3(copy_grid(a.n16)), dim3(256), 0,
                      (cudaStream_t)stream, a);
}

void* fg_mailbox_slot(void* mailbox, int world, int nslot, size_t slot_bytes, int src, int slot) {
  if (!mailbox || world <= 0 || nslot <= 0 || src < 0 || src >= world || slot < 0 || slot >= nslot ||
      slot_bytes == 0 || slot_bytes % 16)
    return nullptr;
  const fg::handoff::Geometry g(world, nslot, slot_bytes);
  return static_cast<uint8_t*>(mailbox) + g.data + ((size_t)src * nslot + slot) * slot_bytes;
}

int fg_handoff_signal(void* my_mailbox, void* peer_mailbox, int world, int me, int dst, size_t slot_bytes,
                      fg_stream_t stream) {
  using namespace fg::handoff;
  FG_REQUIRE(my_mailbox && peer_mailbox, "fg_handoff_signal: null pointer");
  FG_REQUIRE(world > 0 && me >= 0 && me < world && dst >= 0 && dst < world && dst != me,
             "fg_handoff_signal: bad ranks me=%d dst=%d world=%d", me, dst, world);
  const Geometry g(world, 1, slot_bytes);
  uint32_t* peer_flag = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(peer_mailbox) + g.flags) +
                        (size_t)me * kWordStride;
  uint32_t* my_send_seq = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(my_mailbox) + g.send_seq) +
                          (size_t)dst * kWordStride;
  return fg::launch_k("fg_handoff_signal", signal_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream,
                      peer_flag, my_send_seq);
}

int fg_handoff_wait(void* my_mailbox, int world, int me, int src, size_t slot_bytes, int timeout_ms,
                    fg_stream_t stream) {
  using namespace fg::handoff;
  FG_REQUIRE(my_mailbox, "fg_handoff_wait: null pointer");
  FG_REQUIRE(world > 0 && me >= 0 && me < world && src >= 0 && src < world && src != me,
             "fg_handoff_wait: bad ranks me=%d src=%d world=%d", me, src, world);
  const Geometry g(world, 1, slot_bytes);
  uint8_t* mine = static_cast<uint8_t*>(my_mailbox);
  const uint32_t* my_flag = reinterpret_cast<const uint32_t*>(mine + g.flags) + (size_t)src * kWordStride;
  uint32_t* my_recv_seq = reinterpret_cast<uint32_t*>(mine + g.recv_seq) + (size_t)src * kWordStride;
  const uint64_t timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
  return fg::launch_k("fg_handoff_wait", wait_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, my_flag,
                      my_recv_seq, timeout_ns);
}

}  // extern "C"
