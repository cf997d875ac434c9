// Tensor-parallel SUM all-reduce over NVLink peer memory, fused with the
// residual add that follows it in Nebula's decode step:
//
//   out = round(round(sum_r part_r) + residual)      (residual optional)
//
// which is ParallelContext.all_reduce (src/nebula/parallel.py:112-116, a SUM
// over the TP group) followed by the `x = x + part` of
// src/nebula/runtime.py:146,154, each rounded to the model dtype.
//
// Every rank owns a symmetric buffer (peer_layout.cuh), opened by its peers
// through CUDA IPC.  Two low-latency (LL) protocols move the message: each
// 4-byte word travels with the call's epoch in one 8-byte store, so a reader
// polls the words themselves (no fence, no flag round trip):
//   one-shot  every rank pushes its whole partial to every peer and sums all
//             ranks' words locally (one NVLink hop, (W-1) copies out);
//   two-shot  reduce-scatter to sub-shard owners, then all-gather of the
//             finished words (two hops, 2 (W-1)/W of the message out).
// Both sum the ranks in rank order in fp32, so all ranks hold bit-identical
// results.  Epochs live in the buffer (one counter per CTA index, advanced by
// the CTA itself), so a launch recorded in a CUDA graph stays correct on
// replay.  Every wait is bounded (the context's timeout); on expiry the
// kernel raises DEV_ERR_AR_TIMEOUT in the device error word and finishes.
//
// The buffer also carries the exchange region of the all-reduce fused into
// the decode GEMM's epilogue (gemm.cu).
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"

#include "peer_layout.cuh"

namespace fml {
namespace ar {

using peer::Ctx;
using peer::kMaxWorld;
constexpr int kBlocks = peer::kArBlocks;  // fixed grid (one chunk per CTA index, every call)
constexpr int kThreads = 256;
using Args = peer::View;

template <typename T>
__device__ __forceinline__ void add_vec(float (&acc)[16 / sizeof(T)], const uint4& raw) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < (int)(16 / sizeof(T)); ++i) acc[i] += to_f32<T>(e[i]);
}

// Low-latency (LL) variant.  Each 4-byte word of a rank's partial travels
// with the launch's epoch in one 8-byte store, (epoch << 32) | word, into
// slot `rank` of every peer's LL region; a reader polls the pairs of its
// chunk until every epoch matches, so neither a system fence nor a separate
// flag round trip sits on the critical path (8-byte aligned accesses are
// single-copy atomic).  Sums, rounding and the two buffer sets by epoch
// parity are those of ar_kernel.  A reader issues the loads of every peer's
// words of a vector before it checks any of them, so one memory latency, not
// one per peer, precedes the sum.
//
// Reuse of a buffer set.  The grid is always kBlocks CTAs, so after N calls
// every CTA index's epoch is N on every rank and a call's epoch parity is the
// same in all its CTAs.  Call N writes set N&1 of a peer.  Before any write,
// every CTA of call N has passed griddepcontrol.wait, so this rank's call
// N-1 has completed; in it CTA 0 (whose chunk is never empty) read words of
// every peer's call N-1, and each peer wrote those only after its own
// griddepcontrol.wait, i.e. after the peer's call N-2 -- the last reader of
// set N&1 -- had completed.  Sizes may change from call to call.
__device__ __forceinline__ void st_volatile_v2u64(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_volatile_v2u64(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Four (epoch, word) pairs = one 16-byte vector of the message.
__device__ __forceinline__ void ll_load(const uint64_t* p, uint64_t (&w)[4]) {
  ld_volatile_v2u64(p, w[0], w[1]);
  ld_volatile_v2u64(p + 2, w[2], w[3]);
}
__device__ __forceinline__ bool ll_ready(const uint64_t (&w)[4], uint32_t e) {
  return ((uint32_t)(w[0] >> 32) == e) & ((uint32_t)(w[1] >> 32) == e) & ((uint32_t)(w[2] >> 32) == e) &
         ((uint32_t)(w[3] >> 32) == e);
}
// Re-reads the pairs at p until all four carry epoch e (bounded: on expiry
// raises DEV_ERR_AR_TIMEOUT and clears ok, after which nothing waits).
__device__ __forceinline__ void ll_settle(const uint64_t* p, uint64_t (&w)[4], uint32_t e, long long budget,
                                          bool& ok) {
  if (!ok || ll_ready(w, e)) return;
  const long long t0 = clock64();
  while (true) {
    ll_load(p, w);
    if (ll_ready(w, e)) return;
    if (clock64() - t0 > budget) {
      raise_device_error(DEV_ERR_AR_TIMEOUT);
      ok = false;
      return;
    }
  }
}
__device__ __forceinline__ void ll_store(uint64_t* p, uint64_t tag, const uint4& v) {
  st_volatile_v2u64(p, tag | v.x, tag | v.y);
  st_volatile_v2u64(p + 2, tag | v.z, tag | v.w);
}
__device__ __forceinline__ uint4 ll_words(const uint64_t (&w)[4]) {
  return make_uint4((uint32_t)w[0], (uint32_t)w[1], (uint32_t)w[2], (uint32_t)w[3]);
}

// out vector = round(round(sum) + residual) of one 16-byte vector.
template <typename T>
__device__ __forceinline__ uint4 finish_vec(const float (&acc)[16 / sizeof(T)], const T* residual, long long i) {
  constexpr int VE = 16 / sizeof(T);
  float res[VE];
  if (residual != nullptr) {
    const uint4 rv = reinterpret_cast<const uint4*>(residual)[i];
    const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
    for (int k = 0; k < VE; ++k) res[k] = to_f32<T>(re[k]);
  }
  uint4 o;
  T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int k = 0; k < VE; ++k) {
    float x = to_f32<T>(from_f32<T>(acc[k]));  // the all-reduced partial in the model dtype
    if (residual != nullptr) x = x + res[k];   // x + part, rounded once more below
    oe[k] = from_f32<T>(x);
  }
  return o;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) ar_ll_kernel(const __grid_constant__ Args a, const T* __restrict__ part,
                                                         const T* __restrict__ residual, T* __restrict__ out,
                                                         long long nvec) {
  constexpr int VE = 16 / sizeof(T);
  pdl_wait();
  pdl_trigger();
  const int blk = blockIdx.x, tid = threadIdx.x;
  const int W = a.lay.world, r = a.rank;
  uint32_t* epochs = reinterpret_cast<uint32_t*>(a.base[r] + a.lay.ll_epoch_off(0));
  __shared__ uint32_t s_epoch;
  if (tid == 0) s_epoch = epochs[blk] + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int set = (int)(e & 1u);
  const uint64_t tag = (uint64_t)e << 32;
  const long long per = (nvec + kBlocks - 1) / kBlocks;
  const long long v0 = (long long)blk * per, v1 = min(nvec, v0 + per);
  const uint4* src = reinterpret_cast<const uint4*>(part);
  // 1. push this chunk into slot r of every peer (16 data bytes -> 32 LL bytes)
  for (long long i = v0 + tid; i < v1; i += kThreads) {
    const uint4 v = src[i];
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r) ll_store(reinterpret_cast<uint64_t*>(a.base[q] + a.lay.ll_data_off(set, r)) + 4 * i, tag, v);
  }
  // 2. gather every rank's words of this chunk, sum in rank order, add the residual
  bool ok = true;
  for (long long i = v0 + tid; i < v1; i += kThreads) {
    uint64_t w[kMaxWorld][4];
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r) ll_load(reinterpret_cast<const uint64_t*>(a.base[r] + a.lay.ll_data_off(set, q)) + 4 * i, w[q]);
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r)
        ll_settle(reinterpret_cast<const uint64_t*>(a.base[r] + a.lay.ll_data_off(set, q)) + 4 * i, w[q], e,
                  a.timeout_cycles, ok);
    float acc[VE];
#pragma unroll
    for (int k = 0; k < VE; ++k) acc[k] = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W) add_vec<T>(acc, q == r ? src[i] : ll_words(w[q]));
    reinterpret_cast<uint4*>(out)[i] = finish_vec<T>(acc, residual, i);
  }
  __syncthreads();
  if (tid == 0) epochs[blk] = e;
}

// Two-shot LL variant for larger groups: chunk b (one per CTA index) is cut
// into `world` contiguous sub-shards, sub-shard q owned by rank q.
//   1. reduce-scatter: each rank sends every vector it does not own to the
//      owner's area (slot = sender), as (epoch << 32) | word pairs;
//   2. the owner polls the other ranks' words of its vectors, sums all ranks
//      in rank order in fp32 (the one-shot kernels' arithmetic, so results
//      are bit-identical), adds the residual, writes its output and sends the
//      finished 16-bit words to every rank's all-gather area (one writer per
//      position);
//   3. every rank polls the all-gather words of the vectors it does not own.
// A rank sends 2 (W-1)/W of the message (x2 for the pairs) instead of W-1
// copies, for one more NVLink hop.  No wait precedes a send that another rank
// waits for (sends of step 1 come first; step 2's sends need only step 1's
// data), so the steps cannot deadlock.  Buffer-set reuse follows the
// one-shot kernel's argument: every output vector of chunk 0 in call N-1 is
// a sum of words that every rank wrote in call N-1 after its
// griddepcontrol.wait (directly for the owner, through the owner's
// all-gather words for the others), so each peer's call N-2 had completed
// before this rank's call N-1 could finish.
template <typename T>
__global__ void __launch_bounds__(kThreads) ar_ts_kernel(const __grid_constant__ Args a, const T* __restrict__ part,
                                                         const T* __restrict__ residual, T* __restrict__ out,
                                                         long long nvec) {
  constexpr int VE = 16 / sizeof(T);
  pdl_wait();
  pdl_trigger();
  const int blk = blockIdx.x, tid = threadIdx.x;
  const int W = a.lay.world, r = a.rank;
  uint32_t* epochs = reinterpret_cast<uint32_t*>(a.base[r] + a.lay.ts_epoch_off(0));
  __shared__ uint32_t s_epoch;
  if (tid == 0) s_epoch = epochs[blk] + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int set = (int)(e & 1u);
  const uint64_t tag = (uint64_t)e << 32;
  const long long per = (nvec + kBlocks - 1) / kBlocks;
  const long long v0 = (long long)blk * per, v1 = min(nvec, v0 + per);
  const long long len = v1 - v0;
  const uint4* src = reinterpret_cast<const uint4*>(part);
  auto owner = [&](long long i) { return (int)(((i - v0) * W) / len); };
  // 1. reduce-scatter sends
  for (long long i = v0 + tid; i < v1; i += kThreads) {
    const int o = owner(i);
    if (o == r) continue;
    ll_store(reinterpret_cast<uint64_t*>(a.base[o] + a.lay.ts_rs_off(set, r)) + 4 * i, tag, src[i]);
  }
  bool ok = true;
  // 2. owned vectors: reduce in rank order, add the residual, all-gather sends
  for (long long i = v0 + tid; i < v1; i += kThreads) {
    if (owner(i) != r) continue;
    uint64_t w[kMaxWorld][4];
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r) ll_load(reinterpret_cast<const uint64_t*>(a.base[r] + a.lay.ts_rs_off(set, q)) + 4 * i, w[q]);
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r)
        ll_settle(reinterpret_cast<const uint64_t*>(a.base[r] + a.lay.ts_rs_off(set, q)) + 4 * i, w[q], e,
                  a.timeout_cycles, ok);
    float acc[VE];
#pragma unroll
    for (int k = 0; k < VE; ++k) acc[k] = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W) add_vec<T>(acc, q == r ? src[i] : ll_words(w[q]));
    const uint4 o = finish_vec<T>(acc, residual, i);
    reinterpret_cast<uint4*>(out)[i] = o;
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < W && q != r) ll_store(reinterpret_cast<uint64_t*>(a.base[q] + a.lay.ts_ag_off(set)) + 4 * i, tag, o);
  }
  // 3. all-gather receives
  for (long long i = v0 + tid; i < v1; i += kThreads) {
    if (owner(i) == r) continue;
    const uint64_t* p = reinterpret_cast<const uint64_t*>(a.base[r] + a.lay.ts_ag_off(set)) + 4 * i;
    uint64_t w[4];
    ll_load(p, w);
    ll_settle(p, w, e, a.timeout_cycles, ok);
    reinterpret_cast<uint4*>(out)[i] = ll_words(w);
  }
  __syncthreads();
  if (tid == 0) epochs[blk] = e;
}

// Protocol of a call: the context's choice, else the one-shot.
static int ar_proto(const Ctx* c) { return c->proto != 0 ? c->proto : 1; }

}  // namespace ar
}  // namespace fml

using fml::ar::Ctx;
using fml::ar::kMaxWorld;
using fml::fail;

extern "C" {

int64_t neb_ar_handle_bytes(void) { return (int64_t)sizeof(cudaIpcMemHandle_t); }

int neb_ar_create(int64_t max_bytes, int world, int rank, double timeout_ms, void** ctx_out, void* handle_out) {
  if (!ctx_out || !handle_out) return fail(FML_EINVAL, "neb_ar_create: null pointer");
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return fail(FML_EINVAL, "neb_ar_create: world must be 1..8 and 0 <= rank < world");
  if (max_bytes <= 0 || max_bytes % 16 != 0) return fail(FML_EINVAL, "neb_ar_create: max_bytes must be a positive multiple of 16");
  if (!(timeout_ms > 0)) return fail(FML_EINVAL, "neb_ar_create: timeout must be positive");
  Ctx* c = new Ctx();
  c->v.lay.slot_bytes = max_bytes;
  c->v.lay.nsub = (int)((max_bytes + 1023) / 1024);
  c->proto = 0;
  c->v.lay.world = world;
  c->v.rank = rank;
  int clk_khz = 0;
  c->device = fml::current_device();
  if (cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, c->device) != cudaSuccess || clk_khz <= 0) clk_khz = 2000000;
  c->v.timeout_cycles = (long long)(timeout_ms * (double)clk_khz);
  const long long total = c->v.lay.total();
  cudaError_t e = cudaMalloc(&c->own, (size_t)total);
  if (e != cudaSuccess) { delete c; return fml::check_cuda(e, "neb_ar_create: cudaMalloc"); }
  e = cudaMemset(c->own, 0, (size_t)total);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->own);
  if (e != cudaSuccess) {
    cudaFree(c->own);
    delete c;
    return fml::check_cuda(e, "neb_ar_create: buffer setup");
  }
  std::memcpy(handle_out, &h, sizeof(h));
  for (int q = 0; q < kMaxWorld; ++q) c->v.base[q] = nullptr;
  c->v.base[rank] = c->own;
  *ctx_out = c;
  return FML_OK;
}

// handles: world consecutive IPC handles (neb_ar_handle_bytes() each), as
// returned by neb_ar_create on every rank; this rank's own entry is ignored.
int neb_ar_open(void* ctx, const void* handles) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c || !handles) return fail(FML_EINVAL, "neb_ar_open: null pointer");
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int q = 0; q < c->v.lay.world; ++q) {
    if (q == c->v.rank || c->opened[q]) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, hs[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fml::check_cuda(e, "neb_ar_open: cudaIpcOpenMemHandle");
    c->v.base[q] = static_cast<uint8_t*>(p);
    c->opened[q] = true;
  }
  return FML_OK;
}

// Single-process form: device pointers of every rank's buffer (own entry
// ignored), e.g. buffers of other contexts of this process.  No IPC mapping.
int neb_ar_set_peers(void* ctx, void* const* bases) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c || !bases) return fail(FML_EINVAL, "neb_ar_set_peers: null pointer");
  for (int q = 0; q < c->v.lay.world; ++q) {
    if (q == c->v.rank) continue;
    if (!bases[q]) return fail(FML_EINVAL, "neb_ar_set_peers: null peer buffer");
    c->v.base[q] = static_cast<uint8_t*>(bases[q]);
  }
  return FML_OK;
}

void* neb_ar_buffer(void* ctx) { return ctx ? static_cast<Ctx*>(ctx)->own : nullptr; }

int neb_ar_set_protocol(void* ctx, int protocol) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c) return fail(FML_EINVAL, "neb_ar_set_protocol: null context");
  if (protocol < 0 || protocol > 2) return fail(FML_EINVAL, "neb_ar_set_protocol: protocol must be 0, 1 or 2");
  c->proto = protocol;
  return FML_OK;
}

int neb_ar_all_reduce(void* ctx, const void* part, const void* residual, void* out, int64_t n, int dtype, void* stream) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c || !part || !out) return fail(FML_EINVAL, "neb_ar_all_reduce: null pointer");
  if (!fml::valid_dtype(dtype)) return fail(FML_EINVAL, "neb_ar_all_reduce: bad dtype");
  for (int q = 0; q < c->v.lay.world; ++q)
    if (!c->v.base[q]) return fail(FML_EINVAL, "neb_ar_all_reduce: peers not opened");
  const long long bytes = n * (long long)fml::dtype_size(dtype);
  if (n <= 0 || bytes % 16 != 0) return fail(FML_EUNSUPPORTED, "neb_ar_all_reduce: message must be a positive multiple of 16 bytes");
  if (bytes > c->v.lay.slot_bytes) return fail(FML_EUNSUPPORTED, "neb_ar_all_reduce: message larger than the buffer slot");
  for (const void* p : {part, residual, (const void*)out})
    if (p && reinterpret_cast<uintptr_t>(p) % 16 != 0) return fail(FML_EUNSUPPORTED, "neb_ar_all_reduce: pointers must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long nvec = bytes / 16;
  cudaError_t e;
  const dim3 grid(fml::ar::kBlocks), block(fml::ar::kThreads);
  const bool two_shot = fml::ar::ar_proto(c) == 2;
  if (dtype == FML_F32)
    e = fml::launch_pdl(two_shot ? fml::ar::ar_ts_kernel<float> : fml::ar::ar_ll_kernel<float>, grid, block, 0,
                        st, 1, c->v, static_cast<const float*>(part), static_cast<const float*>(residual),
                        static_cast<float*>(out), nvec);
  else if (dtype == FML_BF16)
    e = fml::launch_pdl(two_shot ? fml::ar::ar_ts_kernel<__nv_bfloat16> : fml::ar::ar_ll_kernel<__nv_bfloat16>,
                        grid, block, 0, st, 1, c->v, static_cast<const __nv_bfloat16*>(part),
                        static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), nvec);
  else
    e = fml::launch_pdl(two_shot ? fml::ar::ar_ts_kernel<__half> : fml::ar::ar_ll_kernel<__half>, grid, block,
                        0, st, 1, c->v, static_cast<const __half*>(part), static_cast<const __half*>(residual),
                        static_cast<__half*>(out), nvec);
  fml::count_launch();
  return fml::check_cuda(e, "neb_ar_all_reduce launch");
}

int neb_ar_destroy(void* ctx) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c) return FML_OK;
  cudaDeviceSynchronize();
  for (int q = 0; q < kMaxWorld; ++q)
    if (c->opened[q] && c->v.base[q]) cudaIpcCloseMemHandle(c->v.base[q]);
  if (c->own) cudaFree(c->own);
  delete c;
  return FML_OK;
}

}  // extern "C"
