// Peer-memory communication over NVLink/NVSwitch for the training ranks.
//
// A *window* is one device allocation per rank, opened in every peer through CUDA
// IPC, so rank r can load from and store to rank p's window at the same offsets
// ("symmetric"). The draft's parameter shards, two full-size gradient slots and a
// flag area live in the window.
//
// Kernels (all waits are bounded: on timeout they set the device error word and
// return; nothing traps or spins forever):
//   peer_allgather   : out[p*ss + i] = window_p[src_off + i]       (pull from every rank;
//                      SM kernel, or copy-engine DMA per shard: peer_allgather_ce)
//   peer_reduce_avg  : grad[i] += bf16( (sum_p window_p[slot + r*ss + i]) / N )
//                      summed in fixed rank order (deterministic)
//   peer_signal/wait : sequence-number flags (release stores to every peer's flag
//                      slot; acquire loads with a poll limit).
#include <cuda_runtime.h>

#include <vector>

#include "common.h"
#include "peer.h"
#include "sm100.cuh"

namespace ns {

// ---------------------------------------------------------------------------- flags
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag area layout (unsigned words at window offset `flags_off`): [channel][source rank].
// signal: every peer p gets flags_p[channel][rank] = seq.
__global__ void peer_signal_kernel(PeerTable t, int64_t flags_off, int channel, int rank, int world, unsigned seq) {
  const int p = threadIdx.x;
  if (p >= world) return;
  __threadfence_system();
  unsigned* f = reinterpret_cast<unsigned*>(t.base[p] + flags_off) + channel * MAX_PEERS + rank;
  st_release_sys(f, seq);
}

// wait until flags_self[channel][p] >= seq for every p (bounded).
__global__ void peer_wait_kernel(PeerTable t, int64_t flags_off, int channel, int rank, int world, unsigned seq,
                                 int* err, long long limit) {
  const int p = threadIdx.x;
  if (p >= world) return;
  const unsigned* f = reinterpret_cast<const unsigned*>(t.base[rank] + flags_off) + channel * MAX_PEERS + p;
  long long i = 0;
  while ((int)(ld_acquire_sys(f) - seq) < 0) {
    if (++i > limit) {
      atomicExch(err, 2);
      return;
    }
    __nanosleep(200);
  }
}

// ---------------------------------------------------------------------------- data movement
// out[p * ss + i] = window_p[src_off + i], i < ss, for every rank p (16-byte chunks).
__global__ void peer_allgather_kernel(PeerTable t, int world, int64_t src_off, int64_t ss_bytes, uint8_t* out) {
  const int64_t chunks = ss_bytes / 16;
  const int64_t total = chunks * world;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / chunks);
    const int64_t c = i % chunks;
    const uint4 v = *reinterpret_cast<const uint4*>(t.base[p] + src_off + c * 16);
    reinterpret_cast<uint4*>(out + p * ss_bytes)[c] = v;
  }
}

// grad[i] = bf16(grad[i] + bf16(sum_p slot_p[rank*ss + i] / world)), fixed p order.
// Each thread keeps U chunks x every peer's 16-byte load in flight before summing
// (remote loads are latency-bound).
constexpr int RED_U = 2;
__global__ void __launch_bounds__(256) peer_reduce_avg_kernel(PeerTable t, int world, int rank, int64_t slot_off,
                                                              int64_t ss, __nv_bfloat16* grad) {
  const int64_t n8 = ss / 8;
  const float inv = 1.f / world;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n8; i0 += RED_U * stride) {
    uint4 v[RED_U][MAX_PEERS];
    uint4 g[RED_U];
#pragma unroll
    for (int u = 0; u < RED_U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n8) {
#pragma unroll
        for (int p = 0; p < MAX_PEERS; ++p)
          if (p < world)
            v[u][p] = *reinterpret_cast<const uint4*>(t.base[p] + slot_off + ((int64_t)rank * ss + i * 8) * 2);
        g[u] = reinterpret_cast<const uint4*>(grad)[i];
      }
    }
#pragma unroll
    for (int u = 0; u < RED_U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n8) break;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int p = 0; p < MAX_PEERS; ++p) {
        if (p >= world) break;
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[u][p]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(h[j]);
      }
      __nv_bfloat16* gh = reinterpret_cast<__nv_bfloat16*>(&g[u]);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        gh[j] = __float2bfloat16(__bfloat162float(gh[j]) + sm100::bf16_round(acc[j] * inv));
      reinterpret_cast<uint4*>(grad)[i] = g[u];
    }
  }
}

// Second half of the copy-engine reduce: the peers' contributions to this rank's
// shard were copied by DMA into `staging` ([world][ss], row `rank` unused); sum
// them with this rank's own slot range in fixed rank order (the same order and
// rounding as peer_reduce_avg_kernel), 8 elements per thread.
__global__ void __launch_bounds__(256) local_reduce_avg_kernel(const __nv_bfloat16* __restrict__ own,
                                                               const __nv_bfloat16* __restrict__ staging,
                                                               int world, int rank, int64_t ss,
                                                               __nv_bfloat16* __restrict__ grad) {
  const int64_t n8 = ss / 8;
  const float inv = 1.f / world;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 v[MAX_PEERS];
#pragma unroll
    for (int p = 0; p < MAX_PEERS; ++p)
      if (p < world)
        v[p] = __ldcs(reinterpret_cast<const uint4*>((p == rank ? own : staging + (int64_t)p * ss)) + i);
    uint4 g = reinterpret_cast<const uint4*>(grad)[i];
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int p = 0; p < MAX_PEERS; ++p) {
      if (p >= world) break;
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[p]);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(h[j]);
    }
    __nv_bfloat16* gh = reinterpret_cast<__nv_bfloat16*>(&g);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      gh[j] = __float2bfloat16(__bfloat162float(gh[j]) + sm100::bf16_round(acc[j] * inv));
    reinterpret_cast<uint4*>(grad)[i] = g;
  }
}

// Element-granularity variants for shard sizes that are not multiples of 8 elements.
__global__ void peer_allgather_scalar_kernel(PeerTable t, int world, int64_t src_off, int64_t ss,
                                             __nv_bfloat16* out) {
  const int64_t total = ss * world;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / ss);
    const int64_t c = i % ss;
    out[i] = reinterpret_cast<const __nv_bfloat16*>(t.base[p] + src_off)[c];
  }
}

__global__ void peer_reduce_avg_scalar_kernel(PeerTable t, int world, int rank, int64_t slot_off, int64_t ss,
                                              __nv_bfloat16* grad) {
  const float inv = 1.f / world;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ss; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int p = 0; p < world; ++p)
      acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(t.base[p] + slot_off)[(int64_t)rank * ss + i]);
    grad[i] = __float2bfloat16(__bfloat162float(grad[i]) + sm100::bf16_round(acc * inv));
  }
}

// ---------------------------------------------------------------------------- one-to-one
// dst window of rank `dst` at byte dst_off <- this rank's src (n16 16-byte chunks).
__global__ void peer_put_kernel(PeerTable t, int dst, int64_t dst_off, const uint4* __restrict__ src, int64_t n16) {
  uint64_t base = t.base[0];
#pragma unroll
  for (int i = 1; i < MAX_PEERS; ++i) base = dst == i ? t.base[i] : base;
  uint4* out = reinterpret_cast<uint4*>(base + dst_off);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = src[i];
  __threadfence_system();  // the stores reach `dst` before a later signal
}

// flags_dst[channel][rank] = seq (one destination).
__global__ void peer_signal_to_kernel(PeerTable t, int64_t flags_off, int channel, int rank, int dst, unsigned seq) {
  if (threadIdx.x != 0) return;
  uint64_t base = t.base[0];
#pragma unroll
  for (int i = 1; i < MAX_PEERS; ++i) base = dst == i ? t.base[i] : base;
  __threadfence_system();
  st_release_sys(reinterpret_cast<unsigned*>(base + flags_off) + channel * MAX_PEERS + rank, seq);
}

// wait until flags_self[channel][src] >= seq (bounded).
__global__ void peer_wait_from_kernel(PeerTable t, int64_t flags_off, int channel, int rank, int src, unsigned seq,
                                      int* err, long long limit) {
  if (threadIdx.x != 0) return;
  uint64_t base = t.base[0];
#pragma unroll
  for (int i = 1; i < MAX_PEERS; ++i) base = rank == i ? t.base[i] : base;
  const unsigned* f = reinterpret_cast<const unsigned*>(base + flags_off) + channel * MAX_PEERS + src;
  long long i = 0;
  while ((int)(ld_acquire_sys(f) - seq) < 0) {
    if (++i > limit) {
      atomicExch(err, 2);
      return;
    }
    __nanosleep(200);
  }
}

// ============================================================================ host
struct Window {
  void* ptr = nullptr;
  int64_t bytes = 0;
  int rank = 0, world = 1;
  PeerTable table{};
  std::vector<void*> opened;
};

static std::vector<Window*> g_windows;

// Allocates this rank's window and returns (handle id, IPC handle bytes).
std::vector<int64_t> window_create(int64_t bytes, int64_t rank, int64_t world) {
  NS_CHECK(world <= MAX_PEERS, "peer windows support up to 8 ranks");
  auto* w = new Window();
  w->bytes = (bytes + (2 << 20) - 1) / (2 << 20) * (2 << 20);
  w->rank = (int)rank;
  w->world = (int)world;
  NS_CUDA(cudaMalloc(&w->ptr, w->bytes));
  NS_CUDA(cudaMemset(w->ptr, 0, w->bytes));
  g_windows.push_back(w);
  return {(int64_t)(g_windows.size() - 1), (int64_t)reinterpret_cast<uintptr_t>(w->ptr)};
}

at::Tensor window_ipc_handle(int64_t id) {
  Window* w = g_windows.at(id);
  cudaIpcMemHandle_t h;
  NS_CUDA(cudaIpcGetMemHandle(&h, w->ptr));
  auto t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

// handles: [world, 64] uint8 (CPU); opens every peer's window.
void window_open(int64_t id, at::Tensor handles) {
  Window* w = g_windows.at(id);
  NS_CHECK(handles.size(0) == w->world, "one IPC handle per rank expected");
  for (int p = 0; p < w->world; ++p) {
    if (p == w->rank) {
      w->table.base[p] = reinterpret_cast<uint64_t>(w->ptr);
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handles[p].data_ptr(), sizeof(h));
    void* ptr = nullptr;
    NS_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    w->opened.push_back(ptr);
    w->table.base[p] = reinterpret_cast<uint64_t>(ptr);
  }
}

void window_close(int64_t id) {
  Window* w = g_windows.at(id);
  if (!w) return;
  NS_CUDA(cudaDeviceSynchronize());
  for (void* p : w->opened) NS_CUDA(cudaIpcCloseMemHandle(p));
  w->opened.clear();
  if (w->ptr) NS_CUDA(cudaFree(w->ptr));
  w->ptr = nullptr;
  delete w;
  g_windows[id] = nullptr;
}

WindowInfo window_info(int64_t id) {
  NS_CHECK(id >= 0 && id < (int64_t)g_windows.size() && g_windows[id], "peer window is not open");
  const Window* w = g_windows[id];
  return {w->table, w->rank, w->world, w->bytes};
}

// A tensor view of this rank's window (bytes [offset, offset + numel*itemsize)).
at::Tensor window_view(int64_t id, int64_t offset, int64_t numel, at::ScalarType dtype) {
  Window* w = g_windows.at(id);
  const int64_t item = at::elementSize(dtype);
  NS_CHECK(offset % 16 == 0 && offset + numel * item <= w->bytes, "window view out of range or misaligned");
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  return at::from_blob(static_cast<uint8_t*>(w->ptr) + offset, {numel},
                       at::TensorOptions().dtype(dtype).device(at::kCUDA, dev));
}

static int blocks_for(int64_t items) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)num_sms() * 4));
}

// All-gather on the copy engines: one peer-to-peer cudaMemcpyAsync per rank's shard
// (NVLink DMA, no SMs taken from the overlapped compute).
void peer_allgather_ce(int64_t id, int64_t src_off, int64_t ss_elems, at::Tensor out) {
  Window* w = g_windows.at(id);
  const int64_t ss_bytes = ss_elems * 2;
  NS_CHECK(out.numel() * out.element_size() >= ss_bytes * w->world, "all-gather output too small");
  uint8_t* dst = static_cast<uint8_t*>(out.data_ptr());
  for (int p = 0; p < w->world; ++p)
    NS_CUDA(cudaMemcpyAsync(dst + p * ss_bytes, reinterpret_cast<const void*>(w->table.base[p] + src_off), ss_bytes,
                            cudaMemcpyDeviceToDevice, stream()));
}

void peer_allgather(int64_t id, int64_t src_off, int64_t ss_elems, at::Tensor out) {
  Window* w = g_windows.at(id);
  const int64_t ss_bytes = ss_elems * 2;
  NS_CHECK(src_off % 16 == 0, "peer all-gather needs a 16-byte aligned source");
  NS_CHECK(out.numel() * out.element_size() >= ss_bytes * w->world, "all-gather output too small");
  if (ss_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 != 0) {
    peer_allgather_scalar_kernel<<<blocks_for(ss_elems * w->world), 256, 0, stream()>>>(
        w->table, w->world, src_off, ss_elems, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
    NS_CUDA(cudaGetLastError());
    return;
  }
  peer_allgather_kernel<<<blocks_for(ss_bytes / 16 * w->world), 256, 0, stream()>>>(
      w->table, w->world, src_off, ss_bytes, static_cast<uint8_t*>(out.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

void peer_reduce_avg(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad) {
  Window* w = g_windows.at(id);
  NS_CHECK(slot_off % 16 == 0, "peer reduce needs a 16-byte aligned slot");
  if (ss_elems % 8 != 0 || reinterpret_cast<uintptr_t>(grad.data_ptr()) % 16 != 0) {
    peer_reduce_avg_scalar_kernel<<<blocks_for(ss_elems), 256, 0, stream()>>>(
        w->table, w->world, w->rank, slot_off, ss_elems, reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
    NS_CUDA(cudaGetLastError());
    return;
  }
  peer_reduce_avg_kernel<<<blocks_for(ss_elems / 8), 256, 0, stream()>>>(
      w->table, w->world, w->rank, slot_off, ss_elems, reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

// Reduce on the copy engines: DMA every peer's range [rank*ss, (rank+1)*ss) of its
// gradient slot into `staging` ([world][ss] bf16), then one local kernel sums the
// contributions in rank order into `grad`. NVLink traffic takes no SMs.
void peer_reduce_avg_ce(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad, at::Tensor staging) {
  Window* w = g_windows.at(id);
  NS_CHECK(slot_off % 16 == 0, "peer reduce needs a 16-byte aligned slot");
  NS_CHECK(staging.numel() >= ss_elems * w->world, "reduce staging buffer too small");
  const int64_t bytes = ss_elems * 2;
  auto* st = static_cast<uint8_t*>(staging.data_ptr());
  for (int p = 0; p < w->world; ++p) {
    if (p == w->rank) continue;
    NS_CUDA(cudaMemcpyAsync(st + p * bytes, reinterpret_cast<const void*>(w->table.base[p] + slot_off + w->rank * bytes),
                            bytes, cudaMemcpyDeviceToDevice, stream()));
  }
  const auto* own = reinterpret_cast<const __nv_bfloat16*>(w->table.base[w->rank] + slot_off + w->rank * bytes);
  if (ss_elems % 8 != 0 || reinterpret_cast<uintptr_t>(grad.data_ptr()) % 16 != 0 || (w->rank * bytes) % 16 != 0) {
    // unaligned shards: the SM pull kernel reads the same values
    peer_reduce_avg(id, slot_off, ss_elems, grad);
    return;
  }
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((ss_elems / 8 + 255) / 256, (int64_t)num_sms() * 2));
  local_reduce_avg_kernel<<<blocks, 256, 0, stream()>>>(own, reinterpret_cast<const __nv_bfloat16*>(st), w->world,
                                                        w->rank, ss_elems,
                                                        reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

// Reduce after pushes: every rank stored its contribution to this rank's shard into
// row p (p = its rank) of this rank's slot ([world][ss] bf16, local memory), so the
// sum reads only local memory, in the same rank order and rounding as the pull paths.
void peer_reduce_local(int64_t id, int64_t slot_off, int64_t ss_elems, at::Tensor grad) {
  Window* w = g_windows.at(id);
  NS_CHECK(slot_off % 16 == 0 && ss_elems % 8 == 0 && reinterpret_cast<uintptr_t>(grad.data_ptr()) % 16 == 0,
           "push-mode reduce needs 16-byte aligned shards");
  NS_CHECK(grad.numel() >= ss_elems, "gradient shard too small");
  const auto* slot = reinterpret_cast<const __nv_bfloat16*>(w->table.base[w->rank] + slot_off);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((ss_elems / 8 + 255) / 256, (int64_t)num_sms() * 2));
  local_reduce_avg_kernel<<<blocks, 256, 0, stream()>>>(slot + (int64_t)w->rank * ss_elems, slot, w->world, w->rank,
                                                        ss_elems, reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

// Copies `src` (16-byte aligned, a multiple of 16 bytes) into rank `dst`'s window at
// byte `dst_off`, by SM stores over NVLink.
void peer_put(int64_t id, int64_t dst, int64_t dst_off, at::Tensor src) {
  Window* w = g_windows.at(id);
  const int64_t bytes = src.numel() * src.element_size();
  NS_CHECK(src.is_contiguous() && bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0 &&
               dst_off % 16 == 0,
           "peer_put: 16-byte aligned contiguous source and destination expected");
  NS_CHECK(dst >= 0 && dst < w->world, "peer_put: destination rank outside the window's world");
  if (bytes == 0) return;
  peer_put_kernel<<<blocks_for(bytes / 16), 256, 0, stream()>>>(w->table, (int)dst, dst_off,
                                                                reinterpret_cast<const uint4*>(src.data_ptr()),
                                                                bytes / 16);
  NS_CUDA(cudaGetLastError());
}

void peer_signal_to(int64_t id, int64_t flags_off, int64_t channel, int64_t dst, int64_t seq) {
  Window* w = g_windows.at(id);
  NS_CHECK(dst >= 0 && dst < w->world, "peer_signal_to: destination rank outside the window's world");
  peer_signal_to_kernel<<<1, 32, 0, stream()>>>(w->table, flags_off, (int)channel, w->rank, (int)dst, (unsigned)seq);
  NS_CUDA(cudaGetLastError());
}

void peer_wait_from(int64_t id, int64_t flags_off, int64_t channel, int64_t src, int64_t seq, int64_t poll_limit) {
  Window* w = g_windows.at(id);
  NS_CHECK(src >= 0 && src < w->world, "peer_wait_from: source rank outside the window's world");
  peer_wait_from_kernel<<<1, 32, 0, stream()>>>(w->table, flags_off, (int)channel, w->rank, (int)src, (unsigned)seq,
                                               device_error_flag(), (long long)poll_limit);
  NS_CUDA(cudaGetLastError());
}

void peer_signal(int64_t id, int64_t flags_off, int64_t channel, int64_t seq) {
  Window* w = g_windows.at(id);
  peer_signal_kernel<<<1, 32, 0, stream()>>>(w->table, flags_off, (int)channel, w->rank, w->world, (unsigned)seq);
  NS_CUDA(cudaGetLastError());
}

void peer_wait(int64_t id, int64_t flags_off, int64_t channel, int64_t seq, int64_t poll_limit) {
  Window* w = g_windows.at(id);
  peer_wait_kernel<<<1, 32, 0, stream()>>>(w->table, flags_off, (int)channel, w->rank, w->world, (unsigned)seq,
                                          device_error_flag(), (long long)poll_limit);
  NS_CUDA(cudaGetLastError());
}

}  // namespace ns
