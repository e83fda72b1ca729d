// Expert parallelism over NVLink peer memory: dispatch, remote expert products and combine of
// the MoE block (laguna_mlx/laguna.py:147-150) with experts sharded over W GPUs of one node.
// The reference runs on one device and has no counterpart; BASELINE config 5 defines the split.
//
// Every rank owns the contiguous experts [r*El, (r+1)*El) and one "arena" of device memory that
// its peers map (CUDA IPC, plain peer pointers). Per forward, with an epoch e (the same on every
// rank: given by the host, or held on the device and advanced by lg_ep_advance after each
// forward, so that a forward can be replayed from a CUDA graph):
//  1. ep_plan_kernel      per destination rank d, the source's tokens with a pick on d get
//                         consecutive slots in token order (one CTA per d, block scans);
//  2. ep_dispatch_kernel  one warp per (token, d): the token's row, its k expert ids local to
//                         d (-1 where a pick is elsewhere), its k routing weights and its index
//                         go straight into d's arena (16-byte peer stores, only the rows that
//                         exist cross NVLink); the last CTA publishes the row count and then
//                         flags dispatch[src] = e in every peer (release, system scope);
//  3. ep_recv_kernel      the owner waits (bounded) for every source's flag, then marks the
//                         slots past each source's count as carrying no pick;
//  4. expert products     the grouped tcgen05 / GEMV kernels over the received rows; the down
//                         epilogue writes bf16(bf16(y) * w) of every pick straight into the
//                         source's combine rows at (token * k + j) (peer stores) and fences;
//  5. ep_signal_kernel    flags combine[owner] = e in every peer;
//  6. ep_combine_kernel   the source waits (bounded) for every owner's flag, then sums each
//                         token's k rows in pick order: bf16(bf16(bf16(sum) * scale) + shared),
//                         the arithmetic of the one-GPU combine, so the result is bit-identical
//                         to the one-GPU block on the same tokens.
// Buffer reuse is safe across forwards: a source writes into an owner's receive rows for
// forward e + 1 only after its own combine of forward e, which waited for that owner's combine
// flag, which the owner raised after it had read the rows of forward e.
// Waits give up after a caller-given time; the status word of the arena then records which
// wait expired and the forward completes with wrong values instead of hanging the GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "moe.cuh"

namespace lg {

constexpr int EP_MAX_W = 8;

// arena header: u32 words at fixed offsets
constexpr size_t EP_HDR = 4096;
constexpr size_t EPH_DISPATCH = 0;     // [W] epoch of the last dispatch received from each src
constexpr size_t EPH_COMBINE = 64;     // [W] epoch of the last combine rows from each owner
constexpr size_t EPH_COUNT = 128;      // [W] rows received from each src
constexpr size_t EPH_STATUS = 192;     // status word (0 = ok)
constexpr size_t EPH_DONE = 256;       // CTA completion counter of this rank's dispatch
constexpr size_t EPH_SENDCNT = 320;    // [W] rows this rank sends to each owner
constexpr size_t EPH_EPOCH = 384;      // forwards this rank has completed (device-held epochs)

struct EpLayout {
  size_t recv_x, recv_lid, recv_w, recv_tok, ret, slot, total;
};

static EpLayout ep_layout(int W, int Tr, int k, int H) {
  size_t used = EP_HDR;
  auto take = [&](size_t bytes) {
    used = align_up(used, 256);
    const size_t o = used;
    used += bytes;
    return o;
  };
  EpLayout L;
  const size_t R = (size_t)W * Tr;
  L.recv_x = take(R * H * 2);
  L.recv_lid = take(R * k * 4);
  L.recv_w = take(R * k * 2);
  L.recv_tok = take(R * 4);
  L.ret = take(((size_t)Tr * k + Tr) * H * 2);
  L.slot = take((size_t)Tr * W * 4);
  L.total = align_up(used, 256);
  return L;
}

struct EpPeers {
  char* arena[EP_MAX_W];
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned* hdr_u32(char* arena, size_t off) {
  return reinterpret_cast<unsigned*>(arena + off);
}

// Waits until flags[s] >= epoch for every s < W (bounded); returns false on expiry after
// recording `code` in the status word. Called by one thread.
__device__ bool ep_wait_flags(char* arena, size_t flags_off, int W, unsigned epoch,
                              unsigned long long timeout_ns, unsigned code) {
  const unsigned* f = hdr_u32(arena, flags_off);
  const unsigned long long t0 = globaltimer_ns();
  for (int s = 0; s < W; ++s) {
    while ((int)(ld_acquire_sys(f + s) - epoch) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(hdr_u32(arena, EPH_STATUS), 0u, code | ((unsigned)s << 8));
        return false;
      }
      __nanosleep(256);
    }
  }
  return true;
}

// The epoch of this forward: the caller's, or for epoch 0 one past the forwards this rank has
// completed, as counted on the device by ep_advance_kernel. Device-held epochs let a forward be
// captured once in a CUDA graph and replayed; every rank replays the same number of forwards,
// so the ranks' counters agree.
__device__ __forceinline__ unsigned ep_epoch(char* self, unsigned epoch) {
  return epoch ? epoch : *reinterpret_cast<volatile unsigned*>(hdr_u32(self, EPH_EPOCH)) + 1u;
}

__device__ __forceinline__ bool ep_owns(int e, int El, int W, int d) {
  return e >= 0 && e < El * W && e / El == d;
}

// Expert placement: owner[e] (the rank holding expert e) and local[e] (its index among that
// rank's El experts), or null for the contiguous ranges (owner e / El, local e % El).
struct EpMap {
  const int32_t* owner;
  const int32_t* local;
};

__device__ __forceinline__ bool ep_owns_m(const EpMap& m, int e, int El, int W, int d) {
  if (!m.owner) return ep_owns(e, El, W, d);
  return e >= 0 && e < El * W && __ldg(m.owner + e) == d;
}

__device__ __forceinline__ int ep_local_m(const EpMap& m, int e, int El, int d) {
  return m.owner ? __ldg(m.local + e) : e - d * El;
}

// One CTA per destination rank d: tokens with at least one pick on d take consecutive slots
// (token order); slot[t * W + d] = -1 for the others; the total goes to the send count.
__global__ void __launch_bounds__(512) ep_plan_kernel(const int32_t* __restrict__ inds, int T,
                                                      int k, int El, int W, char* self,
                                                      EpLayout L, EpMap map) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_total;
  const int d = blockIdx.x;
  int32_t* slot = reinterpret_cast<int32_t*>(self + L.slot);
  int base = 0;
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    int has = 0;
    if (t < T)
      for (int j = 0; j < k; ++j) has |= ep_owns_m(map, inds[(size_t)t * k + j], El, W, d);
    const int off = block_excl_scan(has, warp_tot, &s_total);
    if (t < T) slot[(size_t)t * W + d] = has ? base + off : -1;
    base += s_total;
  }
  if (threadIdx.x == 0) hdr_u32(self, EPH_SENDCNT)[d] = (unsigned)base;
}

// One warp per (token, destination): the row, the k local expert ids (-1 for picks owned
// elsewhere), the k routing weights and the token index, stored into the owner's arena.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const int32_t* __restrict__ inds,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          int T, int Tr, int H, int k, int El,
                                                          int W, int rank, EpPeers peers,
                                                          EpLayout L, unsigned epoch, EpMap map) {
  pdl_wait();
  pdl_trigger();
  char* self = peers.arena[rank];
  epoch = ep_epoch(self, epoch);
  const int lane = threadIdx.x & 31;
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int nw = (int)((gridDim.x * blockDim.x) >> 5);
  const int32_t* slot = reinterpret_cast<const int32_t*>(self + L.slot);
  const int nvec = H / 8;
  for (int item = gw; item < T * W; item += nw) {
    const int t = item / W, d = item - t * W;
    const int s = slot[(size_t)t * W + d];
    if (s < 0) continue;  // the whole warp holds the same item
    char* dst = peers.arena[d];
    const size_t row = (size_t)rank * Tr + s;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
    uint4* drow = reinterpret_cast<uint4*>(dst + L.recv_x) + row * nvec;
    for (int v = lane; v < nvec; v += 32) drow[v] = src[v];
    if (lane < k) {
      const int e = inds[(size_t)t * k + lane];
      reinterpret_cast<int32_t*>(dst + L.recv_lid)[row * k + lane] =
          ep_owns_m(map, e, El, W, d) ? ep_local_m(map, e, El, d) : -1;
      reinterpret_cast<__nv_bfloat16*>(dst + L.recv_w)[row * k + lane] = w[(size_t)t * k + lane];
    }
    if (lane == 0) reinterpret_cast<int32_t*>(dst + L.recv_tok)[row] = t;
  }
  __threadfence_system();  // this thread's peer stores before the CTA counts itself done
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* done = hdr_u32(self, EPH_DONE);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {  // the last CTA publishes counts, then flags
      __threadfence_system();
      const unsigned* sendcnt = hdr_u32(self, EPH_SENDCNT);
      for (int d = 0; d < W; ++d)
        *reinterpret_cast<volatile unsigned*>(hdr_u32(peers.arena[d], EPH_COUNT) + rank) =
            sendcnt[d];
      __threadfence_system();
      for (int d = 0; d < W; ++d) st_release_sys(hdr_u32(peers.arena[d], EPH_DISPATCH) + rank, epoch);
      *done = 0;
    }
  }
}

// The owner: wait for every source's dispatch of this epoch, then give the slots past each
// source's row count no picks (their contents are left from earlier forwards).
__global__ void __launch_bounds__(256) ep_recv_kernel(char* self, int W, int Tr, int k,
                                                      unsigned epoch,
                                                      unsigned long long timeout_ns,
                                                      EpLayout L) {
  pdl_wait();
  pdl_trigger();
  __shared__ int ok;
  __shared__ unsigned cnt[EP_MAX_W];
  if (threadIdx.x == 0) {
    ok = ep_wait_flags(self, EPH_DISPATCH, W, ep_epoch(self, epoch), timeout_ns, 1u);
    for (int s = 0; s < W; ++s) cnt[s] = ok ? ld_acquire_sys(hdr_u32(self, EPH_COUNT) + s) : 0u;
  }
  __syncthreads();
  int32_t* lid = reinterpret_cast<int32_t*>(self + L.recv_lid);
  const size_t n = (size_t)W * Tr * k;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / k;
    const int s = (int)(row / Tr), sl = (int)(row - (size_t)s * Tr);
    if (sl >= (int)cnt[s]) lid[i] = -1;
  }
}

// The owner, after its expert products: flag combine[owner] = epoch in every source.
__global__ void ep_signal_kernel(EpPeers peers, int W, int rank, unsigned epoch) {
  epoch = ep_epoch(peers.arena[rank], epoch);
  __threadfence_system();
  if ((int)threadIdx.x < W) st_release_sys(hdr_u32(peers.arena[threadIdx.x], EPH_COMBINE) + rank, epoch);
}

// The source: wait for every owner's rows of this epoch, then per token the one-GPU combine of
// the k weighted pick rows (already bf16(y * w)) in pick order, the routed scale and the shared
// expert's row.
__global__ void __launch_bounds__(256) ep_combine_kernel(char* self, int W, int T, int Tr, int k,
                                                         int E, int H,
                                                         const int32_t* __restrict__ inds,
                                                         float scale, int has_shared,
                                                         unsigned epoch,
                                                         unsigned long long timeout_ns,
                                                         EpLayout L,
                                                         __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ int ok;
  if (threadIdx.x == 0)
    ok = ep_wait_flags(self, EPH_COMBINE, W, ep_epoch(self, epoch), timeout_ns, 2u);
  __syncthreads();
  const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(self + L.ret);
  const __nv_bfloat16* sh = y + (size_t)Tr * k * H;
  const int H8 = H / 8;
  const size_t total = (size_t)T * H8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / H8;
    const int c = (int)(i % H8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int e = inds[t * k + j];
      if (e < 0 || e >= E) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(y + (t * k + j) * H + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += __uint_as_float(u[q] << 16);
        acc[2 * q + 1] += __uint_as_float(u[q] & 0xFFFF0000u);
      }
    }
    float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (has_shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(sh + t * H + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        s8[2 * q] = __uint_as_float(u[q] << 16);
        s8[2 * q + 1] = __uint_as_float(u[q] & 0xFFFF0000u);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float r0 = round_bf16(round_bf16(acc[2 * q]) * scale);
      float r1 = round_bf16(round_bf16(acc[2 * q + 1]) * scale);
      if (has_shared) {
        r0 += s8[2 * q];
        r1 += s8[2 * q + 1];
      }
      if (!ok) r0 = r1 = __int_as_float(0x7fc00000);  // a wait expired: the values are unknown
      __nv_bfloat162 b = __floats2bfloat162_rn(r0, r1);
      o[q] = *reinterpret_cast<uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(out + t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// After a forward's combine (stream order): this rank has completed one more forward.
__global__ void ep_advance_kernel(char* self) {
  if (threadIdx.x == 0) *hdr_u32(self, EPH_EPOCH) += 1u;
}

}  // namespace lg

using namespace lg;

namespace {

int ep_check(int W, int rank, int Tr, int k, int H) {
  LG_CHECK_ARG(W >= 1 && W <= EP_MAX_W && rank >= 0 && rank < W,
               "ep: %d ranks (at most %d), rank %d", W, EP_MAX_W, rank);
  LG_CHECK_ARG(Tr >= 1 && k >= 1 && k <= 32 && H > 0 && H % 8 == 0,
               "ep: capacity %d tokens, k=%d, hidden %d (a multiple of 8)", Tr, k, H);
  return LG_OK;
}

int ep_peers(void* const* arenas, int W, EpPeers* p) {
  LG_CHECK_ARG(arenas != nullptr, "ep: NULL arena table");
  for (int d = 0; d < EP_MAX_W; ++d) {
    p->arena[d] = d < W ? static_cast<char*>(arenas[d]) : nullptr;
    if (d < W) LG_CHECK_ARG(p->arena[d] && aligned(p->arena[d], 256), "ep: arena %d is NULL or "
                                                                       "not 256-byte aligned", d);
  }
  return LG_OK;
}

unsigned long long ep_timeout_ns(double s) {
  return s > 0 ? (unsigned long long)(s * 1e9) : 2000000000ull;
}

}  // namespace

extern "C" size_t lg_ep_arena_bytes(int W, int Tr, int k, int H) {
  if (W < 1 || W > EP_MAX_W || Tr < 1 || k < 1 || H <= 0) return 0;
  return ep_layout(W, Tr, k, H).total;
}

extern "C" int lg_ep_arena_offsets(int W, int Tr, int k, int H, size_t* shared_rows,
                                   size_t* combine_rows) {
  LG_CHECK_ARG(shared_rows && combine_rows, "ep_arena_offsets: NULL output");
  const EpLayout L = ep_layout(W, Tr, k, H);
  *combine_rows = L.ret;
  *shared_rows = L.ret + (size_t)Tr * k * H * 2;
  return LG_OK;
}

extern "C" int lg_ep_ipc_handle(const void* ptr, void* handle, size_t* offset) {
  LG_CHECK_ARG(ptr && handle && offset, "ep_ipc_handle: NULL pointer");
  static PFN_cuMemGetAddressRange_v3020 range = nullptr;
  if (!range) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess)
      return fail(LG_ERR_CUDA, "ep_ipc_handle: cuMemGetAddressRange unavailable");
    range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(LG_ERR_INVALID, "ep_ipc_handle: %p is not device memory", ptr);
  cudaIpcMemHandle_t h;
  LG_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base;
  return LG_OK;
}

extern "C" size_t lg_ep_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int lg_ep_ipc_open(const void* handle, size_t offset, void** ptr, void** base) {
  LG_CHECK_ARG(handle && ptr && base, "ep_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  LG_CUDA_TRY(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess));
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return LG_OK;
}

extern "C" int lg_ep_ipc_close(void* base) {
  LG_CHECK_ARG(base, "ep_ipc_close: NULL pointer");
  LG_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return LG_OK;
}

extern "C" int lg_ep_dispatch_mapped(const void* x, const int32_t* inds, const void* weights,
                                     int T, int Tr, int H, int k, int E, int W, int rank,
                                     void* const* arenas, unsigned epoch,
                                     const int32_t* owner_of, const int32_t* local_of,
                                     void* stream) {
  if (int rc = ep_check(W, rank, Tr, k, H)) return rc;
  LG_CHECK_ARG(T >= 0 && T <= Tr, "ep_dispatch: %d tokens exceed the capacity %d", T, Tr);
  LG_CHECK_ARG(E >= W && E % W == 0, "ep_dispatch: %d experts do not split over %d ranks", E, W);
  LG_CHECK_ARG(T == 0 || (x && inds && weights && aligned(x, 16)),
               "ep_dispatch: NULL or misaligned x/inds/weights");
  LG_CHECK_ARG(!owner_of == !local_of, "ep_dispatch: owner and local maps go together");
  EpPeers peers;
  if (int rc = ep_peers(arenas, W, &peers)) return rc;
  const EpLayout L = ep_layout(W, Tr, k, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const EpMap map = {owner_of, local_of};
  LG_CUDA_TRY(launch_k(ep_plan_kernel, dim3(W), dim3(512), 0, st, inds, T, k, E / W, W,
                       peers.arena[rank], L, map));
  LG_LAUNCH_CHECK("ep_plan");
  int grid = (T * W + 7) / 8;  // 8 warps per CTA
  if (grid > 148 * 8) grid = 148 * 8;
  if (grid < 1) grid = 1;
  LG_CUDA_TRY(launch_k(ep_dispatch_kernel, dim3(grid), dim3(256), 0, st,
                       static_cast<const __nv_bfloat16*>(x), inds,
                       static_cast<const __nv_bfloat16*>(weights), T, Tr, H, k, E / W, W, rank,
                       peers, L, epoch, map));
  LG_LAUNCH_CHECK("ep_dispatch");
  return LG_OK;
}

extern "C" int lg_ep_dispatch(const void* x, const int32_t* inds, const void* weights, int T,
                              int Tr, int H, int k, int E, int W, int rank,
                              void* const* arenas, unsigned epoch, void* stream) {
  return lg_ep_dispatch_mapped(x, inds, weights, T, Tr, H, k, E, W, rank, arenas, epoch, nullptr,
                               nullptr, stream);
}

extern "C" size_t lg_ep_experts_workspace_bytes(int W, int Tr, int H, int I, int El, int k) {
  if (W < 1 || Tr < 1 || H <= 0 || I <= 0 || El < 1 || k < 1) return 0;
  return moe_ep_workspace_bytes(W * Tr, H, I, El, k);
}

extern "C" int lg_ep_experts(int W, int Tr, int H, int I, int El, int k, const uint32_t* gate_q,
                             const void* gate_s, const void* gate_b, const uint32_t* up_q,
                             const void* up_s, const void* up_b, const uint32_t* down_q,
                             const void* down_s, const void* down_b, int rank,
                             void* const* arenas, unsigned epoch, double timeout_s, int path,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = ep_check(W, rank, Tr, k, H)) return rc;
  LG_CHECK_ARG(k <= El * W, "ep_experts: k=%d exceeds the %d experts", k, El * W);
  EpPeers peers;
  if (int rc = ep_peers(arenas, W, &peers)) return rc;
  const EpLayout L = ep_layout(W, Tr, k, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* self = peers.arena[rank];
  const size_t n = (size_t)W * Tr * k;
  int grid = (int)((n + 255) / 256);
  if (grid > 148 * 4) grid = 148 * 4;
  LG_CUDA_TRY(launch_k(ep_recv_kernel, dim3(grid), dim3(256), 0, st, self, W, Tr, k, epoch,
                       ep_timeout_ns(timeout_s), L));
  LG_LAUNCH_CHECK("ep_recv");
  EpRet ep = {};
  for (int d = 0; d < W; ++d)
    ep.ret[d] = reinterpret_cast<__nv_bfloat16*>(peers.arena[d] + L.ret);
  ep.tok = reinterpret_cast<const int32_t*>(self + L.recv_tok);
  ep.w = reinterpret_cast<const __nv_bfloat16*>(self + L.recv_w);
  ep.Tr = Tr;
  ep.on = 1;
  const uint32_t* q[3] = {gate_q, up_q, down_q};
  const void* s[3] = {gate_s, up_s, down_s};
  const void* b[3] = {gate_b, up_b, down_b};
  int rc = moe_experts_ep(self + L.recv_x, W * Tr, H, I, El, k,
                          reinterpret_cast<const int32_t*>(self + L.recv_lid), ep.w, q, s, b,
                          path, workspace, workspace_bytes, ep, st);
  if (rc) return rc;
  ep_signal_kernel<<<1, 32, 0, st>>>(peers, W, rank, epoch);
  LG_LAUNCH_CHECK("ep_signal");
  return LG_OK;
}

extern "C" int lg_ep_combine(const int32_t* inds, int T, int Tr, int H, int k, int E,
                             float routed_scale, int has_shared, int W, int rank,
                             void* const* arenas, unsigned epoch, double timeout_s, void* out,
                             void* stream) {
  if (int rc = ep_check(W, rank, Tr, k, H)) return rc;
  LG_CHECK_ARG(T >= 0 && T <= Tr, "ep_combine: %d tokens exceed the capacity %d", T, Tr);
  LG_CHECK_ARG(T == 0 || (inds && out && aligned(out, 16)), "ep_combine: NULL inds/out");
  EpPeers peers;
  if (int rc = ep_peers(arenas, W, &peers)) return rc;
  const EpLayout L = ep_layout(W, Tr, k, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t n = (size_t)T * (H / 8);
  int grid = (int)((n + 255) / 256);
  if (grid > 148 * 8) grid = 148 * 8;
  if (grid < 1) grid = 1;
  LG_CUDA_TRY(launch_k(ep_combine_kernel, dim3(grid), dim3(256), 0, st, peers.arena[rank], W, T,
                       Tr, k, E, H, inds, routed_scale, has_shared, epoch,
                       ep_timeout_ns(timeout_s), L, static_cast<__nv_bfloat16*>(out)));
  LG_LAUNCH_CHECK("ep_combine");
  return LG_OK;
}

extern "C" int lg_ep_advance(void* arena, void* stream) {
  LG_CHECK_ARG(arena && aligned(arena, 256), "ep_advance: NULL or misaligned arena");
  ep_advance_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<char*>(arena));
  LG_LAUNCH_CHECK("ep_advance");
  return LG_OK;
}

extern "C" int lg_ep_status(const void* arena, int reset, int* status) {
  LG_CHECK_ARG(arena && status, "ep_status: NULL pointer");
  unsigned v = 0;
  unsigned* p = reinterpret_cast<unsigned*>(static_cast<char*>(const_cast<void*>(arena)) +
                                            EPH_STATUS);
  LG_CUDA_TRY(cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost));
  if (reset && v) LG_CUDA_TRY(cudaMemset(p, 0, sizeof(v)));
  *status = (int)v;
  return LG_OK;
}
