// In-kernel NVLink collectives over a symmetric IPC heap, sm_100a.
//
// Symmetric memory: every rank cudaMalloc's a buffer of the same size, exports a CUDA IPC handle,
// and opens its peers' handles (host code in parallel/symm.py exchanges the 64-byte handles through
// torch.distributed). Kernels then read and write peers' memory with ordinary 16-byte ld/st over
// NVLink / NVSwitch (P2P). No NVLS object is created and no TMA is used here.
//
// Synchronisation: each rank owns a signal pad (int32 per peer) in symmetric memory. A barrier with
// epoch e has rank r store e (st.release.sys) into pad_j[r] of every peer j and then spin (bounded by
// a wall-clock budget, ld.acquire.sys) until its own pad_r[j] >= e for all j. Epochs grow
// monotonically, so pads never need resetting. A timed-out wait records BRAIN_ERR_TIMEOUT_PEER in
// the status word and returns; the host raises. Collectives are phases separated by barriers:
//   all_reduce (two-shot): barrier, reduce-scatter chunk r from all peers into own chunk r, barrier,
//                          all-gather chunk j from peer j;  (one-shot for small: every rank reduces
//                          the whole vector from all peers into its output)
//   reduce_scatter, all_gather, broadcast: one barrier, then pull from peers.
//   fused DDP step (ddp_step): pull every rank's gradient for this rank's shard, sum in f32, scale,
//                          AdamW on the f32 master shard, write the bf16 weights locally and push
//                          them into every peer's parameter buffer; a closing barrier publishes them.
// Reference: ring_allreduce_simulate (crates/brain-distributed/src/collective/allreduce.rs:35-121)
// sums p in-process "ranks"; DataParallel averages (data_parallel.rs:32-70); AdamW order as in
// crates/brain-optim/src/adam/mod.rs:128-200.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kMaxRanks = 8;

struct Peers {
  void* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// One warp: thread j signals peer j and waits for peer j's signal.
__global__ void barrier_kernel(Peers pads, int rank, int world, int epoch, int64_t budget_ns, int where) {
  const int j = threadIdx.x;
  if (j >= world) return;
  __threadfence_system();
  int* remote = reinterpret_cast<int*>(pads.p[j]) + rank;
  st_release_sys(remote, epoch);
  const int* mine = reinterpret_cast<const int*>(pads.p[rank]) + j;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(mine) < epoch) {
    if (globaltimer() - t0 > (uint64_t)budget_ns) {
      set_status(BRAIN_ERR_TIMEOUT_PEER, where * 16 + j);
      return;
    }
  }
}

template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};

__device__ __forceinline__ void ld_vec(const float* p, float* f) {
  float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
__device__ __forceinline__ void st_vec(float* p, const float* f) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
__device__ __forceinline__ void ld_vec(const __nv_bfloat16* p, float* f) { load8(p, f); }
__device__ __forceinline__ void st_vec(__nv_bfloat16* p, const float* f) { store8(p, f); }

// out[i] = scale * sum_j peer_j[src_off + i] for i in [0, n); n multiple of the vector width.
template <typename T>
__global__ void reduce_pull_kernel(Peers src, int64_t src_off, int world, int first, T* __restrict__ out, int64_t n,
                                   float scale) {
  constexpr int V = Vec<T>::N;
  const int64_t nv = n / V;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    for (int jj = 0; jj < world; ++jj) {
      const int j = (first + jj) % world;  // stagger peers so ranks do not all hit the same one
      float x[V];
      ld_vec(reinterpret_cast<const T*>(src.p[j]) + src_off + i * V, x);
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] += x[k];
    }
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] *= scale;
    st_vec(out + i * V, acc);
  }
}

// Small- and mid-size all-reduce in one launch. CTA c owns vectors [c * per, (c + 1) * per) (the last CTA
// also the scalar tail when n is not a whole number of vectors): it copies them from `in` into this rank's
// staging (half `parity` of the symmetric buffer), publishes flag c to every rank with a system-scope release
// store of `epoch`, waits until every rank's flag c carries `epoch`, then sums its part of all ranks' staging
// into `out` (which may alias `in`). The staging is double-buffered by call parity: a rank can only begin
// the call after next once every peer has entered the next call, i.e. has finished reading this one, so one
// signal phase per call suffices. This needs each rank's calls to execute in issue order (one stream, or the
// host orders a stream switch). Every rank sums the ranks' copies in the same order (rank 0 first), so the
// results agree bitwise. flags: peer j's int32 [kOneShotCtas][kMaxRanks].
constexpr int kOneShotCtas = 128;
template <typename T>
__global__ void oneshot_allreduce_kernel(const T* in, T* out, int64_t n, Peers stage, Peers flags, int rank, int world,
                                         int epoch, int64_t budget_ns, float scale) {
  constexpr int V = Vec<T>::N;
  const int64_t nv = n / V;
  const int64_t per = (nv + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per, v1 = v0 + per < nv ? v0 + per : nv;
  const bool tail_cta = blockIdx.x == gridDim.x - 1;
  T* mine = reinterpret_cast<T*>(stage.p[rank]);
  for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x)
    *reinterpret_cast<uint4*>(mine + i * V) = *reinterpret_cast<const uint4*>(in + i * V);
  if (tail_cta)
    for (int64_t e = nv * V + threadIdx.x; e < n; e += blockDim.x) mine[e] = in[e];
  __syncthreads();
  if (threadIdx.x < world) {
    const int j = threadIdx.x;
    __threadfence_system();
    st_release_sys(reinterpret_cast<int*>(flags.p[j]) + blockIdx.x * kMaxRanks + rank, epoch);
    const int* f = reinterpret_cast<const int*>(flags.p[rank]) + blockIdx.x * kMaxRanks + j;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer() - t0 > (uint64_t)budget_ns) {
        set_status(BRAIN_ERR_TIMEOUT_PEER, 1200 + j);
        break;
      }
    }
  }
  __syncthreads();
  for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
    float acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    for (int j = 0; j < world; ++j) {
      float x[V];
      ld_vec(reinterpret_cast<const T*>(stage.p[j]) + i * V, x);
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] += x[k];
    }
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] *= scale;
    st_vec(out + i * V, acc);
  }
  if (tail_cta)
    for (int64_t e = nv * V + threadIdx.x; e < n; e += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < world; ++j) acc += static_cast<float>(reinterpret_cast<const T*>(stage.p[j])[e]);
      out[e] = static_cast<T>(acc * scale);
    }
}

// Mid- and large-size all-reduce in one launch (reduce-scatter + all-gather, two signal phases). The vector
// is split into `world` shards; CTA c owns slice c of every shard (the same element positions on every
// rank). Phase A: copy this CTA's slices of `in` into this rank's staging, signal flag c (epoch e1), wait for
// every rank's flag c. Phase B: sum slice c of shard `rank` over all ranks' staging (rank 0 first), scale,
// and store the result into that position of every rank's staging (only this rank reads or writes shard
// `rank` there), signal flag c (epoch e1 + 1), wait for every rank's flag c. Phase C: copy this CTA's
// slices of all shards from the staging into `out` (which may alias `in`). A rank starts its next call only
// after all its CTAs saw every peer finish phase B, so one staging buffer is enough. flags: int32 [128][8].
template <typename T>
__global__ void twoshot_allreduce_kernel(const T* in, T* out, int64_t n, Peers stage, Peers flags, int rank,
                                         int world, int e1, int64_t budget_ns, float scale) {
  constexpr int V = Vec<T>::N;
  const int64_t S = n / world;  // shard length (a whole number of vectors)
  const int64_t nvs = S / V;
  const int64_t per = (nvs + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per, v1 = v0 + per < nvs ? v0 + per : nvs;
  T* mine = reinterpret_cast<T*>(stage.p[rank]);
  for (int s = 0; s < world; ++s)
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x)
      *reinterpret_cast<uint4*>(mine + s * S + i * V) = *reinterpret_cast<const uint4*>(in + s * S + i * V);
  for (int phase = 0; phase < 2; ++phase) {
    __syncthreads();
    if (threadIdx.x < world) {
      const int j = threadIdx.x;
      __threadfence_system();
      st_release_sys(reinterpret_cast<int*>(flags.p[j]) + blockIdx.x * kMaxRanks + rank, e1 + phase);
      const int* f = reinterpret_cast<const int*>(flags.p[rank]) + blockIdx.x * kMaxRanks + j;
      const uint64_t t0 = globaltimer();
      while (ld_acquire_sys(f) < e1 + phase) {
        if (globaltimer() - t0 > (uint64_t)budget_ns) {
          set_status(BRAIN_ERR_TIMEOUT_PEER, 1300 + phase * 16 + j);
          break;
        }
      }
    }
    __syncthreads();
    if (phase == 0) {
      const int64_t base = rank * S;
      for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
        float acc[V];
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] = 0.f;
        for (int j = 0; j < world; ++j) {
          float x[V];
          ld_vec(reinterpret_cast<const T*>(stage.p[j]) + base + i * V, x);
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k] += x[k];
        }
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] *= scale;
        for (int jj = 0; jj < world; ++jj) {
          const int j = (rank + jj) % world;  // stagger the pushes so ranks do not all hit one peer
          st_vec(reinterpret_cast<T*>(stage.p[j]) + base + i * V, acc);
        }
      }
    }
  }
  for (int s = 0; s < world; ++s)
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x)
      *reinterpret_cast<uint4*>(out + s * S + i * V) = *reinterpret_cast<const uint4*>(mine + s * S + i * V);
}

// dst[dst_off + i] = peer_src[src_off + i]  (copy of n elements, 16-byte vectors)
__global__ void copy_pull_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t nbytes) {
  const int64_t nv = nbytes / 16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x)
    reinterpret_cast<int4*>(dst)[i] = reinterpret_cast<const int4*>(src)[i];
}

// all-gather pull: for every peer j != rank, copy bytes [j*chunk, (j+1)*chunk) of peer j's buffer
// into the same range of the local buffer (blockIdx.y selects the peer).
__global__ void gather_pull_kernel(Peers bufs, int rank, int world, int64_t chunk_bytes, int64_t base_off) {
  const int j = (rank + 1 + blockIdx.y) % world;
  if (j == rank) return;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(bufs.p[j]) + base_off + j * chunk_bytes;
  uint8_t* dst = reinterpret_cast<uint8_t*>(bufs.p[rank]) + base_off + j * chunk_bytes;
  const int64_t nv = chunk_bytes / 16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x)
    reinterpret_cast<int4*>(dst)[i] = reinterpret_cast<const int4*>(src)[i];
}

// all-gather push: copy bytes [rank*chunk, (rank+1)*chunk) of the local buffer into the same range of every
// peer's buffer (blockIdx.y selects the peer). Remote stores need no round trip, so four 16-byte vectors
// per thread are in flight at once. The caller orders it: no peer may still use that range (a barrier, or a
// protocol step after which nobody reads it) before, and a barrier after it publishes the data.
__global__ void gather_push_kernel(Peers bufs, int rank, int world, int64_t chunk_bytes, int64_t base_off) {
  const int j = (rank + 1 + blockIdx.y) % world;
  if (j == rank) return;
  const int4* src = reinterpret_cast<const int4*>(reinterpret_cast<const uint8_t*>(bufs.p[rank]) + base_off +
                                                  rank * chunk_bytes);
  int4* dst = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(bufs.p[j]) + base_off + rank * chunk_bytes);
  const int64_t nv = chunk_bytes / 16;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (; i + 3 * stride < nv; i += 4 * stride) {
    const int4 a = src[i], b = src[i + stride], c = src[i + 2 * stride], d = src[i + 3 * stride];
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < nv; i += stride) dst[i] = src[i];
}

// Fused data-parallel optimizer step over this rank's shard [off, off + n):
//   g = grad_scale * sum_j grad_j[off + i]       (pull over NVLink, f32 accumulate)
//   AdamW (decay, moments, bias-corrected update) on the f32 master shard
//   w16 = bf16(master) written to every rank's parameter buffer at [off + i] (local + P2P push)
template <typename G>
__global__ void ddp_step_kernel(Peers grads, Peers params, int rank, int world, int pworld, int64_t off, int64_t n,
                                float* __restrict__ master, float* __restrict__ m, float* __restrict__ v, float lr,
                                float b1, float b2, float eps, float wd, float inv_bc1, float inv_bc2,
                                float grad_scale) {
  constexpr int V = 8;  // 8 elements per thread-iteration (16 B of bf16 params)
  const int64_t nv = n / V;
  const float decay = 1.f - lr * wd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * V;
    float g[V];
#pragma unroll
    for (int k = 0; k < V; ++k) g[k] = 0.f;
    for (int jj = 0; jj < world; ++jj) {
      const int j = (rank + jj) % world;
      const G* gp = reinterpret_cast<const G*>(grads.p[j]) + off + e;
      float x[V];
      if constexpr (sizeof(G) == 2) {
        ld_vec(reinterpret_cast<const __nv_bfloat16*>(gp), x);
      } else {
        ld_vec(reinterpret_cast<const float*>(gp), x);
        ld_vec(reinterpret_cast<const float*>(gp) + 4, x + 4);
      }
#pragma unroll
      for (int k = 0; k < V; ++k) g[k] += x[k];
    }
    float pm[V], mm[V], vv[V];
    ld_vec(master + e, pm);
    ld_vec(master + e + 4, pm + 4);
    ld_vec(m + e, mm);
    ld_vec(m + e + 4, mm + 4);
    ld_vec(v + e, vv);
    ld_vec(v + e + 4, vv + 4);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float gg = g[k] * grad_scale;
      pm[k] *= decay;
      mm[k] = b1 * mm[k] + (1.f - b1) * gg;
      vv[k] = b2 * vv[k] + (1.f - b2) * gg * gg;
      pm[k] -= lr * (mm[k] * inv_bc1) / (sqrtf(vv[k] * inv_bc2) + eps);
    }
    st_vec(master + e, pm);
    st_vec(master + e + 4, pm + 4);
    st_vec(m + e, mm);
    st_vec(m + e + 4, mm + 4);
    st_vec(v + e, vv);
    st_vec(v + e + 4, vv + 4);
    bf16x8 w;
#pragma unroll
    for (int k = 0; k < 4; ++k) w.h[k] = __floats2bfloat162_rn(pm[2 * k], pm[2 * k + 1]);
    for (int jj = 0; jj < pworld; ++jj) {
      const int j = (rank + jj) % pworld;
      *reinterpret_cast<bf16x8*>(reinterpret_cast<__nv_bfloat16*>(params.p[j]) + off + e) = w;
    }
  }
}

int grid_for(int64_t work) {
  int64_t g = (work + 255) / 256;
  int64_t cap = (int64_t)brain_host::num_sms() * 4;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

Peers to_peers(const int64_t* ptrs, int world) {
  Peers p{};
  for (int i = 0; i < world && i < kMaxRanks; ++i) p.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return p;
}

}  // namespace

BRAIN_STATUS_READER(comm)

// ---------------------------------------------------------------- symmetric heap (host)
BRAIN_API int brain_ipc_alloc(int64_t bytes, int64_t* ptr_out, void* handle_out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e != cudaSuccess) return (int)e;
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return (int)e;
  }
  *ptr_out = reinterpret_cast<int64_t>(p);
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

BRAIN_API int brain_ipc_handle_size() { return (int)sizeof(cudaIpcMemHandle_t); }

BRAIN_API int brain_ipc_open(const void* handle, int64_t* ptr_out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return (int)e;
  *ptr_out = reinterpret_cast<int64_t>(p);
  return 0;
}

BRAIN_API int brain_ipc_close(int64_t ptr) { return (int)cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

BRAIN_API int brain_ipc_free(int64_t ptr) { return (int)cudaFree(reinterpret_cast<void*>(ptr)); }

// ---------------------------------------------------------------- collectives
// pads: int64[world] peer pointers of the signal pads (each int32[kMaxRanks]).
BRAIN_API int brain_comm_barrier(const int64_t* pads, int rank, int world, int epoch, int64_t budget_ns, int where,
                                 cudaStream_t st) {
  if (world > kMaxRanks) return (int)cudaErrorInvalidValue;
  barrier_kernel<<<1, 32, 0, st>>>(to_peers(pads, world), rank, world, epoch, budget_ns, where);
  return (int)cudaGetLastError();
}

// out[0:n) = scale * sum_j peer_j[src_off : src_off + n)   (dtype: 0 = f32, 1 = bf16)
BRAIN_API int brain_comm_reduce_pull(const int64_t* bufs, int64_t src_off, int rank, int world, void* out, int64_t n,
                                     int dtype, float scale, cudaStream_t st) {
  Peers p = to_peers(bufs, world);
  if (dtype == 0) {
    if (n % 4) return (int)cudaErrorInvalidValue;
    reduce_pull_kernel<float><<<grid_for(n / 4), 256, 0, st>>>(p, src_off, world, rank, reinterpret_cast<float*>(out), n,
                                                              scale);
  } else {
    if (n % 8) return (int)cudaErrorInvalidValue;
    reduce_pull_kernel<__nv_bfloat16><<<grid_for(n / 8), 256, 0, st>>>(p, src_off, world, rank,
                                                                      reinterpret_cast<__nv_bfloat16*>(out), n, scale);
  }
  return (int)cudaGetLastError();
}

// local[base + j*chunk, ...) = peer_j[base + j*chunk, ...) for all j != rank.
BRAIN_API int brain_comm_gather_pull(const int64_t* bufs, int rank, int world, int64_t chunk_bytes, int64_t base_off,
                                     cudaStream_t st) {
  if (chunk_bytes % 16 || base_off % 16) return (int)cudaErrorInvalidValue;
  if (world <= 1) return 0;
  dim3 grid(std::max(1, grid_for(chunk_bytes / 16) / (world - 1)), world - 1);
  gather_pull_kernel<<<grid, 256, 0, st>>>(to_peers(bufs, world), rank, world, chunk_bytes, base_off);
  return (int)cudaGetLastError();
}

// peer_j[base + rank*chunk, ...) = local[base + rank*chunk, ...) for all j != rank (push; see gather_push_kernel).
BRAIN_API int brain_comm_gather_push(const int64_t* bufs, int rank, int world, int64_t chunk_bytes, int64_t base_off,
                                     cudaStream_t st) {
  if (chunk_bytes % 16 || base_off % 16) return (int)cudaErrorInvalidValue;
  if (world <= 1) return 0;
  dim3 grid(std::max(1, grid_for(chunk_bytes / 64) / (world - 1)), world - 1);
  gather_push_kernel<<<grid, 256, 0, st>>>(to_peers(bufs, world), rank, world, chunk_bytes, base_off);
  return (int)cudaGetLastError();
}

// Plain copy (local or peer pointer) of nbytes (multiple of 16).
BRAIN_API int brain_comm_copy(int64_t src, int64_t dst, int64_t nbytes, cudaStream_t st) {
  if (nbytes % 16 || (src | dst) % 16) return (int)cudaErrorInvalidValue;
  if (nbytes == 0) return 0;
  copy_pull_kernel<<<grid_for(nbytes / 16), 256, 0, st>>>(reinterpret_cast<const uint8_t*>(src),
                                                          reinterpret_cast<uint8_t*>(dst), nbytes);
  return (int)cudaGetLastError();
}

// Copy-engine copy (local or peer pointer, one cudaMemcpyAsync): overlaps with kernels on other
// streams without taking SMs.
BRAIN_API int brain_comm_copy_async(int64_t src, int64_t dst, int64_t nbytes, cudaStream_t st) {
  if (nbytes == 0) return 0;
  return (int)cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), (size_t)nbytes,
                              cudaMemcpyDeviceToDevice, st);
}

// Fused reduce-scatter + AdamW + bf16 all-gather push for the shard [off, off + n) of this rank.
// grads/params: int64[world] peer pointers of the flat gradient (bf16 if grad_bf16 else f32) and
// bf16 parameter buffers. n must be a multiple of 8 and off 8-aligned.
BRAIN_API int brain_comm_ddp_step_ctas(const int64_t* grads, const int64_t* params, int grad_bf16, int rank,
                                       int world, int64_t off, int64_t n, float* master, float* m, float* v, float lr,
                                       float b1, float b2, float eps, float wd, float bc1, float bc2, float grad_scale,
                                       int max_ctas, int push_world, cudaStream_t st);

BRAIN_API int brain_comm_ddp_step(const int64_t* grads, const int64_t* params, int grad_bf16, int rank, int world,
                                  int64_t off, int64_t n, float* master, float* m, float* v, float lr, float b1,
                                  float b2, float eps, float wd, float bc1, float bc2, float grad_scale,
                                  cudaStream_t st) {
  return brain_comm_ddp_step_ctas(grads, params, grad_bf16, rank, world, off, n, master, m, v, lr, b1, b2, eps, wd, bc1,
                                  bc2, grad_scale, 0, world, st);
}

// Same step with at most max_ctas CTAs (0 = as many as the work needs, up to 4 per SM): a capped grid
// leaves the SMs to the backward kernels when the step runs on a side stream during backward. The
// updated bf16 weights go to params[0 .. push_world) (push_world = 1: this rank's buffer only, when
// the copy engines publish them).
BRAIN_API int brain_comm_ddp_step_ctas(const int64_t* grads, const int64_t* params, int grad_bf16, int rank,
                                       int world, int64_t off, int64_t n, float* master, float* m, float* v, float lr,
                                       float b1, float b2, float eps, float wd, float bc1, float bc2, float grad_scale,
                                       int max_ctas, int push_world, cudaStream_t st) {
  if (n % 8 || off % 8) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  Peers g = to_peers(grads, world), p = to_peers(params, world);
  int grid = grid_for(n / 8);
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  if (push_world < 1 || push_world > world) return (int)cudaErrorInvalidValue;
  if (grad_bf16)
    ddp_step_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(g, p, rank, world, push_world, off, n, master, m, v, lr, b1,
                                                        b2, eps, wd, 1.f / bc1, 1.f / bc2, grad_scale);
  else
    ddp_step_kernel<float><<<grid, 256, 0, st>>>(g, p, rank, world, push_world, off, n, master, m, v, lr, b1, b2,
                                                eps, wd, 1.f / bc1, 1.f / bc2, grad_scale);

  return (int)cudaGetLastError();
}

// One-launch all-reduce of n elements (dtype 0 = f32, 1 = bf16; any n >= 1; in and out 16-byte aligned, may
// alias). stage: int64[world] peer pointers of this call's staging half (>= n elements each); flags:
// int64[world] peer pointers of the flag arrays (int32 [128][8] each, zeroed once). epoch grows by one per
// call. A peer that does not arrive within budget_ns records BRAIN_ERR_TIMEOUT_PEER.
BRAIN_API int brain_comm_allreduce_oneshot(const void* in, void* out, int64_t n, int dtype, float scale,
                                           const int64_t* stage, const int64_t* flags, int rank, int world, int epoch,
                                           int64_t budget_ns, cudaStream_t st) {
  if (world > kMaxRanks || n < 1) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return (int)cudaErrorInvalidValue;
  const int V = dtype == 0 ? 4 : 8;
  const int64_t nv = n / V;
  // one vector per thread where possible: the time is a few NVLink load latencies per loop trip, so trips
  // (not bytes) set the cost up to 128 CTAs x 256 threads x 16 bytes = 512 KB per trip
  const int ctas = (int)std::max<int64_t>(1, std::min<int64_t>(kOneShotCtas, (nv + 255) / 256));
  Peers sp = to_peers(stage, world), fp = to_peers(flags, world);
  if (dtype == 0)
    oneshot_allreduce_kernel<float><<<ctas, 256, 0, st>>>(reinterpret_cast<const float*>(in),
                                                          reinterpret_cast<float*>(out), n, sp, fp, rank, world, epoch,
                                                          budget_ns, scale);
  else
    oneshot_allreduce_kernel<__nv_bfloat16><<<ctas, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), n, sp, fp, rank, world,
        epoch, budget_ns, scale);
  return (int)cudaGetLastError();
}

// One-launch two-phase all-reduce (dtype 0 = f32, 1 = bf16; n a multiple of world x the 16-byte vector; in,
// out 16-byte aligned, may alias). stage: int64[world] peer pointers of staging buffers of >= n elements;
// flags: int64[world] peer pointers of int32 [128][8] flag arrays (zeroed once, not shared with other
// kernels). e1: this call's first epoch; the call uses e1 and e1 + 1.
BRAIN_API int brain_comm_allreduce_twoshot(const void* in, void* out, int64_t n, int dtype, float scale,
                                           const int64_t* stage, const int64_t* flags, int rank, int world, int e1,
                                           int64_t budget_ns, cudaStream_t st) {
  const int V = dtype == 0 ? 4 : 8;
  if (world > kMaxRanks || world < 1 || n < 1 || n % ((int64_t)world * V)) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return (int)cudaErrorInvalidValue;
  const int64_t nvs = n / world / V;
  const int ctas = (int)std::max<int64_t>(1, std::min<int64_t>(kOneShotCtas, (nvs + 255) / 256));
  Peers sp = to_peers(stage, world), fp = to_peers(flags, world);
  if (dtype == 0)
    twoshot_allreduce_kernel<float><<<ctas, 256, 0, st>>>(reinterpret_cast<const float*>(in),
                                                          reinterpret_cast<float*>(out), n, sp, fp, rank, world, e1,
                                                          budget_ns, scale);
  else
    twoshot_allreduce_kernel<__nv_bfloat16><<<ctas, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(in), reinterpret_cast<__nv_bfloat16*>(out), n, sp, fp, rank, world,
        e1, budget_ns, scale);
  return (int)cudaGetLastError();
}
