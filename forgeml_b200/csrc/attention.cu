// Attention kernels.
//
// 1. neb_attention: Nebula's masked attention over the contiguous per-request
//    KV cache (src/nebula/runtime.py:139-144 plus the prefix torch.stack of
//    src/nebula/cache.py:163-165, which this kernel makes unnecessary: keys
//    are read in place from the cache pool).  Flash-decoding layout: one CTA
//    per (query, key split), a half/whole warp per key row with 16-byte
//    vector loads (8 K and V rows in flight per warp), online softmax in fp32,
//    and the key splits of one query combined through distributed shared
//    memory inside a thread-block cluster (no global scratch).
//    HBM-bound: per query it streams 2 * ctx * D elements.
//
// 2. fml_sdpa: ForgeML's rank-4 scaled-dot-product attention
//    (src/forgeml/ops.py:61-70 -> F.scaled_dot_product_attention) with
//    arbitrary strides (the q/k/v of a fused QKV projection are strided views
//    of one slot), causal or boolean/additive mask.  Flash-attention
//    recurrence on CUDA cores with K/V blocks staged in shared memory; fp32
//    arithmetic throughout so the fp32 graph keeps IEEE-level accuracy.
#include <cfloat>
#include <string>

#include "common.cuh"

namespace fml {
namespace attn {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ===========================================================================
// Nebula attention over the KV pool
// ===========================================================================
constexpr int kAttnWarps = 8;
constexpr int kUnroll = 4;
constexpr int kMaxD = 256;

// One lane's share of a K or V row.  VEC: a raw 16-byte slice at element
// gl*VE (converted on use).  !VEC: elements gl, gl+G, ... as floats.
template <typename T, bool VEC, int VE>
struct RowSlice;
template <typename T, int VE>
struct RowSlice<T, true, VE> {
  uint4 raw;
  __device__ __forceinline__ void load(const T* row, int gl, int, int, bool ok) {
    raw = ok ? __ldg(reinterpret_cast<const uint4*>(row + gl * VE)) : make_uint4(0, 0, 0, 0);
  }
  __device__ __forceinline__ float get(int i) const { return to_f32<T>(reinterpret_cast<const T*>(&raw)[i]); }
};
template <typename T, int VE>
struct RowSlice<T, false, VE> {
  float v[VE];
  __device__ __forceinline__ void load(const T* row, int gl, int G, int D, bool ok) {
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int d = gl + G * i;
      v[i] = (ok && d < D) ? to_f32<T>(row[d]) : 0.f;
    }
  }
  __device__ __forceinline__ float get(int i) const { return v[i]; }
};

// VEC: each lane of a G-lane group owns one 16-byte slice of the D-vector.
// !VEC: each lane owns elements gl, gl+G, ... (scalar loads; odd head sizes).
template <typename T, int G, bool VEC>
__global__ void __launch_bounds__(kAttnWarps * 32, 3)
    neb_attn_kernel(const T* __restrict__ q, long long qs0, long long qs1, long long qs2,
                    const T* __restrict__ kpool, const T* __restrict__ vpool,
                    const int32_t* __restrict__ slot_of, const int32_t* __restrict__ start_pos,
                    T* __restrict__ out, int tq, int H, int D, int max_seq, float scale,
                    int nsplit) {
  constexpr int VE = VEC ? (int)(16 / sizeof(T)) : (G == 32 ? kMaxD / 32 : 1);
  constexpr int KPW = 32 / G;                 // keys per warp-wide load
  __shared__ float sm_o[kAttnWarps][kMaxD];
  __shared__ float sm_ml[kAttnWarps][2];
  __shared__ float res_o[kMaxD];
  __shared__ float res_ml[2];

  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int group = lane / G, gl = lane % G;
  const long long qidx = blockIdx.x / nsplit;
  const int split = (int)(blockIdx.x % nsplit);
  const int h = (int)(qidx % H);
  const int t = (int)((qidx / H) % tq);
  const int b = (int)(qidx / ((long long)H * tq));

  const int slot = slot_of[b];
  const int pos = start_pos[b] + t;  // absolute position of this query
  bool bad = (slot < 0) || (pos < 0) || (pos >= max_seq);
  const int len = bad ? 0 : pos + 1;
  if (bad && split == 0 && threadIdx.x == 0) raise_device_error(DEV_ERR_ATTN_RANGE);
  const int lo = (int)((long long)split * len / nsplit);
  const int hi = (int)((long long)(split + 1) * len / nsplit);

  const long long head_off = ((long long)(bad ? 0 : slot) * H + h) * (long long)max_seq * D;
  const T* kh = kpool + head_off;
  const T* vh = vpool + head_off;
  const T* qp = q + b * qs0 + (long long)t * qs1 + (long long)h * qs2;

  // Query slice, pre-scaled.
  float qv[VE];
  int nel;  // valid elements owned by this lane
  if (VEC) {
    nel = (gl * VE < D) ? VE : 0;
    if (nel) {
      uint4 raw = *reinterpret_cast<const uint4*>(qp + gl * VE);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < VE; ++i) qv[i] = to_f32<T>(e[i]) * scale;
    } else {
#pragma unroll
      for (int i = 0; i < VE; ++i) qv[i] = 0.f;
    }
  } else {
    nel = 0;
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int d = gl + G * i;
      qv[i] = d < D ? to_f32<T>(qp[d]) * scale : 0.f;
      nel += d < D;
    }
  }

  float m = -INFINITY, l = 0.f;
  float o[VE];
#pragma unroll
  for (int i = 0; i < VE; ++i) o[i] = 0.f;

  constexpr int KB = KPW * kUnroll;  // keys per warp iteration
  for (int base = lo + warp * KB; base < hi; base += kAttnWarps * KB) {
    // Issue every load of this iteration before any use; the 16-byte slices
    // stay in raw form and are converted where they are consumed.
    RowSlice<T, VEC, VE> ks[kUnroll], vs[kUnroll];
    bool valid[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int key = base + u * KPW + group;
      valid[u] = key < hi;
      ks[u].load(kh + (long long)key * D, gl, G, D, valid[u] && nel > 0);
      vs[u].load(vh + (long long)key * D, gl, G, D, valid[u] && nel > 0);
    }
    float s[kUnroll];
    float bmax = -INFINITY;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < VE; ++i) d = fmaf(qv[i], ks[u].get(i), d);
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      s[u] = valid[u] ? d : -INFINITY;
      bmax = fmaxf(bmax, s[u]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, off));
    const float m_new = fmaxf(m, bmax);
    const float alpha = expf(m - m_new);  // 0 while m is -inf
    l *= alpha;
#pragma unroll
    for (int i = 0; i < VE; ++i) o[i] *= alpha;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const float pr = expf(s[u] - m_new);
      l += pr;
#pragma unroll
      for (int i = 0; i < VE; ++i) o[i] = fmaf(pr, vs[u].get(i), o[i]);
    }
    m = m_new;
  }
  // Sum the groups of this warp (each group holds distinct keys).
#pragma unroll
  for (int off = 16; off >= G; off >>= 1) {
    l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
    for (int i = 0; i < VE; ++i) o[i] += __shfl_xor_sync(0xffffffffu, o[i], off);
  }
  if (group == 0) {
    if (VEC) {
      if (nel)
#pragma unroll
        for (int i = 0; i < VE; ++i) sm_o[warp][gl * VE + i] = o[i];
    } else {
#pragma unroll
      for (int i = 0; i < VE; ++i) {
        const int d = gl + G * i;
        if (d < D) sm_o[warp][d] = o[i];
      }
    }
    if (gl == 0) { sm_ml[warp][0] = m; sm_ml[warp][1] = l; }
  }
  __syncthreads();
  // Combine the warps of this CTA.
  float mc = -INFINITY;
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) mc = fmaxf(mc, sm_ml[w][0]);
  float lc = 0.f;
  float wgt[kAttnWarps];
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) {
    wgt[w] = (sm_ml[w][0] == -INFINITY) ? 0.f : expf(sm_ml[w][0] - mc);
    lc += wgt[w] * sm_ml[w][1];
  }
  T* op = out + ((long long)b * tq + t) * (long long)H * D + (long long)h * D;
  if (nsplit == 1) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) acc += wgt[w] * sm_o[w][d];
      op[d] = from_f32<T>(bad ? 0.f : acc / lc);
    }
    return;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) acc += wgt[w] * sm_o[w][d];
    res_o[d] = acc;
  }
  if (threadIdx.x == 0) { res_ml[0] = mc; res_ml[1] = lc; }
  cluster_sync_all();
  if (split == 0) {
    const uint32_t a_ml = smem_u32(res_ml), a_o = smem_u32(res_o);
    float mm = -INFINITY;
    for (int r = 0; r < nsplit; ++r) mm = fmaxf(mm, ld_cluster_f32(mapa(a_ml, r)));
    float ww[8];
    float lt = 0.f;
    for (int r = 0; r < nsplit; ++r) {
      const float mr = ld_cluster_f32(mapa(a_ml, r));
      ww[r] = (mr == -INFINITY) ? 0.f : expf(mr - mm);
      lt += ww[r] * ld_cluster_f32(mapa(a_ml + 4, r));
    }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < nsplit; ++r) acc += ww[r] * ld_cluster_f32(mapa(a_o + 4 * d, r));
      op[d] = from_f32<T>(bad ? 0.f : acc / lt);
    }
  }
  cluster_sync_all();  // keep every CTA's shared memory alive until rank 0 has read it
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined variant (16-byte aligned rows).  The keys [lo, hi) of
// one (request, head) are one contiguous run of the pool, so a producer warp
// streams them into shared memory with cp.async.bulk, kBulkStages stages of
// NK keys (a 16 KB K tile plus a 16 KB V tile each) in flight, completion
// signalled as transaction bytes on a per-stage mbarrier.  The K and V copies
// of a stage are issued by two different lanes, and successive stages by
// different lane pairs: one thread's bulk copies complete one after another,
// copies from different threads overlap.  Four consumer warps read the tiles
// with conflict-free 16-byte shared loads (a G-lane group per row, 32/G rows
// per warp-wide load) and run the same online softmax as above; each
// releases a stage back to the producer with one arrive.  Nothing but the
// valid keys is copied, so a ragged final stage needs no bounds on the
// global side.
// ---------------------------------------------------------------------------
constexpr int kBulkConsumers = 4;
// Measured on B200 over 2-6 stages x 8-32 KB tiles: three 16 KB stages
// (two CTAs per SM) stream fastest.
constexpr int kBulkStages = 3;
constexpr int kBulkTile = 16384;  // bytes of one K (or V) tile
constexpr int kBulkSmem = kBulkStages * 2 * kBulkTile;

template <typename T, int G>
__global__ void __launch_bounds__(32 * (kBulkConsumers + 1))
    neb_attn_bulk_kernel(const T* __restrict__ q, long long qs0, long long qs1, long long qs2,
                         const T* __restrict__ kpool, const T* __restrict__ vpool,
                         const int32_t* __restrict__ slot_of, const int32_t* __restrict__ start_pos,
                         T* __restrict__ out, int tq, int H, int D, int max_seq, float scale, int nsplit) {
  constexpr int VE = 16 / (int)sizeof(T);
  constexpr int RB = 16 * G;                    // bytes of one K/V row (= D * sizeof(T))
  constexpr int NK = kBulkTile / RB;            // keys per stage
  constexpr int KPW = 32 / G;                   // rows per warp-wide 16-byte load
  constexpr int KW = NK / kBulkConsumers;       // keys per consumer warp per stage
  constexpr int R = KW / KPW;                   // warp-wide loads per stage (= 8)
  static_assert(R * KPW * kBulkConsumers == NK, "stage split");
  extern __shared__ __align__(1024) uint8_t tiles[];
  __shared__ __align__(8) uint64_t full_bar[kBulkStages], empty_bar[kBulkStages];
  __shared__ float sm_o[kBulkConsumers][kMaxD];
  __shared__ float sm_ml[kBulkConsumers][2];
  __shared__ float res_o[kMaxD];
  __shared__ float res_ml[2];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kBulkConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // slot_of / start_pos are step inputs (never written by this library's
  // kernels), so they may be read before waiting for the previous grid.
  const long long qidx = blockIdx.x / nsplit;
  const int split = (int)(blockIdx.x % nsplit);
  const int h = (int)(qidx % H);
  const int t = (int)((qidx / H) % tq);
  const int b = (int)(qidx / ((long long)H * tq));
  const int slot = slot_of[b];
  const int first_new = start_pos[b];  // rows from here on are this step's (written by the previous grid)
  const int pos = first_new + t;
  const bool bad = (slot < 0) || (pos < 0) || (pos >= max_seq);
  const int len = bad ? 0 : pos + 1;
  if (bad && split == 0 && threadIdx.x == 0) raise_device_error(DEV_ERR_ATTN_RANGE);
  const int lo = (int)((long long)split * len / nsplit);
  const int hi = (int)((long long)(split + 1) * len / nsplit);
  const int nst = (hi - lo + NK - 1) / NK;
  const long long head_off = ((long long)(bad ? 0 : slot) * H + h) * (long long)max_seq * D;
  const uint32_t tiles_u32 = smem_u32(tiles);

  float m = -INFINITY, l = 0.f;
  float o[VE];
#pragma unroll
  for (int i = 0; i < VE; ++i) o[i] = 0.f;
  const int group = lane / G, gl = lane % G;

  if (warp == kBulkConsumers) {
    // Producer warp: lane 0 waits for a free stage and arms its barrier; the
    // stage's K tile is copied by lane 2r and its V tile by lane 2r+1
    // (r = stage index mod 16).  Stage s is reused once all four consumer
    // warps have arrived on empty_bar[s].
    const uint8_t* src = reinterpret_cast<const uint8_t*>((lane & 1) ? vpool : kpool) +
                         (head_off + (long long)lo * D) * (long long)sizeof(T);
    // Stages wholly below first_new hold keys written by earlier steps: the
    // first of them are copied before waiting for the previous grid (the
    // QKV projection that appends this step's rows), hiding one memory
    // latency behind its tail.
    int pre = 0;
    while (pre < nst && pre < kBulkStages && lo + (pre + 1) * NK <= first_new) ++pre;
    int issued = 0;
    for (int j = 0; j < nst; ++j) {
      if (j == pre) {
        pdl_wait();
        pdl_trigger();
      }
      const int s = j % kBulkStages;
      const uint32_t bytes = (uint32_t)min(NK, hi - lo - j * NK) * RB;
      const uint32_t fb = smem_u32(&full_bar[s]);
      bool got = true;
      if (lane == 0) {
        if (j >= kBulkStages)
          got = mbar_wait(smem_u32(&empty_bar[s]), ((j / kBulkStages) - 1) & 1, DEV_ERR_ATTN_TIMEOUT);
        if (got) mbar_arrive_expect_tx(fb, 2 * bytes);
      }
      if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) break;
      if ((lane >> 1) == (j & 15))
        bulk_load(tiles_u32 + s * 2 * kBulkTile + (lane & 1) * kBulkTile, src + (long long)j * kBulkTile, bytes, fb);
      __syncwarp();
      ++issued;
    }
    // Drain: every copy this CTA issued has landed before it may exit (a
    // no-op unless a wait above gave up).
    if (lane == 0)
      for (int j = max(0, issued - kBulkStages); j < issued; ++j)
        mbar_wait(smem_u32(&full_bar[j % kBulkStages]), (j / kBulkStages) & 1, DEV_ERR_ATTN_TIMEOUT);
    if (pre == nst) {
      pdl_wait();
      pdl_trigger();
    }
  } else {
    pdl_wait();
    pdl_trigger();
    // Query slice of this lane, pre-scaled.
    float qv[VE];
    {
      const T* qp = q + b * qs0 + (long long)t * qs1 + (long long)h * qs2;
      uint4 raw = *reinterpret_cast<const uint4*>(qp + gl * VE);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < VE; ++i) qv[i] = to_f32<T>(e[i]) * scale;
    }
    const uint32_t row0 = (uint32_t)(warp * KW + group) * RB + gl * 16;
    for (int j = 0; j < nst; ++j) {
      const int s = j % kBulkStages;
      if (!mbar_wait(smem_u32(&full_bar[s]), (j / kBulkStages) & 1, DEV_ERR_ATTN_TIMEOUT)) break;
      const int nk = min(NK, hi - lo - j * NK);
      const uint8_t* kt = tiles + s * 2 * kBulkTile + row0;
      const uint8_t* vt = kt + kBulkTile;
      uint4 kr[R];
#pragma unroll
      for (int u = 0; u < R; ++u) kr[u] = *reinterpret_cast<const uint4*>(kt + u * KPW * RB);
      float sc[R];
      float bmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const T* e = reinterpret_cast<const T*>(&kr[u]);
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < VE; ++i) d = fmaf(qv[i], to_f32<T>(e[i]), d);
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        const bool valid = warp * KW + u * KPW + group < nk;
        sc[u] = valid ? d : -INFINITY;
        bmax = fmaxf(bmax, sc[u]);
      }
      uint4 vr[R];
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const bool valid = warp * KW + u * KPW + group < nk;
        vr[u] = valid ? *reinterpret_cast<const uint4*>(vt + u * KPW * RB) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, off));
      const float m_new = fmaxf(m, bmax);
      // A warp whose keys of this stage are all past the end keeps m at -inf.
      const float alpha = (m_new == -INFINITY) ? 1.f : expf(m - m_new);
      l *= alpha;
#pragma unroll
      for (int i = 0; i < VE; ++i) o[i] *= alpha;
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const float pr = (sc[u] == -INFINITY) ? 0.f : expf(sc[u] - m_new);
        l += pr;
        const T* e = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
        for (int i = 0; i < VE; ++i) o[i] = fmaf(pr, to_f32<T>(e[i]), o[i]);
      }
      m = m_new;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
    }
    // Sum the row groups of this warp (each group holds distinct keys).
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
      for (int i = 0; i < VE; ++i) o[i] += __shfl_xor_sync(0xffffffffu, o[i], off);
    }
    if (group == 0) {
#pragma unroll
      for (int i = 0; i < VE; ++i) sm_o[warp][gl * VE + i] = o[i];
      if (gl == 0) { sm_ml[warp][0] = m; sm_ml[warp][1] = l; }
    }
  }
  __syncthreads();
  // Combine the consumer warps of this CTA.
  float mc = -INFINITY;
#pragma unroll
  for (int w = 0; w < kBulkConsumers; ++w) mc = fmaxf(mc, sm_ml[w][0]);
  float lc = 0.f;
  float wgt[kBulkConsumers];
#pragma unroll
  for (int w = 0; w < kBulkConsumers; ++w) {
    wgt[w] = (sm_ml[w][0] == -INFINITY) ? 0.f : expf(sm_ml[w][0] - mc);
    lc += wgt[w] * sm_ml[w][1];
  }
  T* op = out + ((long long)b * tq + t) * (long long)H * D + (long long)h * D;
  if (nsplit == 1) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kBulkConsumers; ++w) acc += wgt[w] * sm_o[w][d];
      op[d] = from_f32<T>(bad ? 0.f : acc / lc);
    }
    return;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kBulkConsumers; ++w) acc += wgt[w] * sm_o[w][d];
    res_o[d] = acc;
  }
  if (threadIdx.x == 0) { res_ml[0] = mc; res_ml[1] = lc; }
  cluster_sync_all();
  if (split == 0) {
    const uint32_t a_ml = smem_u32(res_ml), a_o = smem_u32(res_o);
    float mm = -INFINITY;
    for (int r = 0; r < nsplit; ++r) mm = fmaxf(mm, ld_cluster_f32(mapa(a_ml, r)));
    float ww[8];
    float lt = 0.f;
    for (int r = 0; r < nsplit; ++r) {
      const float mr = ld_cluster_f32(mapa(a_ml, r));
      ww[r] = (mr == -INFINITY) ? 0.f : expf(mr - mm);
      lt += ww[r] * ld_cluster_f32(mapa(a_ml + 4, r));
    }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < nsplit; ++r) acc += ww[r] * ld_cluster_f32(mapa(a_o + 4 * d, r));
      op[d] = from_f32<T>(bad ? 0.f : acc / lt);
    }
  }
  cluster_sync_all();
}

template <typename T, int G>
static int launch_neb_bulk(const void* q, const int64_t* qs, const void* kp, const void* vp,
                           const int32_t* slot_of, const int32_t* start_pos, void* out, long long B,
                           long long tq, long long H, long long D, long long max_seq, float scale,
                           int nsplit, cudaStream_t st) {
  static bool attr_set[64] = {};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(neb_attn_bulk_kernel<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kBulkSmem);
    if (e != cudaSuccess) return check_cuda(e, "neb_attention smem attribute");
    attr_set[dev] = true;
  }
  const long long nq = B * tq * H;
  cudaError_t e = launch_pdl(neb_attn_bulk_kernel<T, G>, dim3((unsigned)(nq * nsplit)),
                             dim3(32 * (kBulkConsumers + 1)), kBulkSmem, st, nsplit, static_cast<const T*>(q),
                             (long long)qs[0], (long long)qs[1], (long long)qs[2], static_cast<const T*>(kp),
                             static_cast<const T*>(vp), slot_of, start_pos, static_cast<T*>(out), (int)tq,
                             (int)H, (int)D, (int)max_seq, scale, nsplit);
  count_launch();
  return check_cuda(e, "neb_attention launch");
}

template <typename T, int G, bool VEC>
static int launch_neb(const void* q, const int64_t* qs, const void* kp, const void* vp,
                      const int32_t* slot_of, const int32_t* start_pos, void* out, long long B,
                      long long tq, long long H, long long D, long long max_seq, float scale,
                      int nsplit, cudaStream_t st) {
  const long long nq = B * tq * H;
  cudaError_t e = launch_pdl(neb_attn_kernel<T, G, VEC>, dim3((unsigned)(nq * nsplit)), dim3(kAttnWarps * 32), 0,
                             st, nsplit, static_cast<const T*>(q), (long long)qs[0], (long long)qs[1],
                             (long long)qs[2], static_cast<const T*>(kp), static_cast<const T*>(vp), slot_of,
                             start_pos, static_cast<T*>(out), (int)tq, (int)H, (int)D, (int)max_seq, scale, nsplit);
  count_launch();
  return check_cuda(e, "neb_attention launch");
}

template <typename T>
static int dispatch_neb(const void* q, const int64_t* qs, const void* kp, const void* vp,
                        const int32_t* so, const int32_t* sp, void* out, long long B, long long tq,
                        long long H, long long D, long long ms, float scale, int nsplit,
                        cudaStream_t st) {
  constexpr int VE = 16 / sizeof(T);
  const bool vec_ok = (D % VE == 0) && (qs[2] % VE == 0) && (qs[1] % VE == 0) &&
                      (qs[0] % VE == 0) && (reinterpret_cast<uintptr_t>(q) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(kp) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(vp) % 16 == 0);
  if (vec_ok) {
    const long long nv = D / VE;  // 16-byte slices per row
    // Rows of exactly 16*G bytes stream through the bulk-copy pipeline.
#define NEB_BULK(GG) \
  if (nv == GG) return launch_neb_bulk<T, GG>(q, qs, kp, vp, so, sp, out, B, tq, H, D, ms, scale, nsplit, st);
    NEB_BULK(1) NEB_BULK(2) NEB_BULK(4) NEB_BULK(8) NEB_BULK(16) NEB_BULK(32)
#undef NEB_BULK
#define NEB_CASE(GG) \
  if (nv <= GG) return launch_neb<T, GG, true>(q, qs, kp, vp, so, sp, out, B, tq, H, D, ms, scale, nsplit, st);
    NEB_CASE(1) NEB_CASE(2) NEB_CASE(4) NEB_CASE(8) NEB_CASE(16) NEB_CASE(32)
#undef NEB_CASE
  }
  if (D <= 8) return launch_neb<T, 8, false>(q, qs, kp, vp, so, sp, out, B, tq, H, D, ms, scale, nsplit, st);
  if (D <= 16) return launch_neb<T, 16, false>(q, qs, kp, vp, so, sp, out, B, tq, H, D, ms, scale, nsplit, st);
  return launch_neb<T, 32, false>(q, qs, kp, vp, so, sp, out, B, tq, H, D, ms, scale, nsplit, st);
}

// ===========================================================================
// ForgeML SDPA (CUDA cores, fp32 math)
// ===========================================================================
constexpr int kSdpaThreads = 128;
constexpr int kSdpaBK = 32;       // keys per shared-memory block
constexpr int kSliceMax = 32;     // dims per thread

struct SdpaParams {
  const void *q, *k, *v, *mask;
  long long qs[4], ks[4], vs[4], ms[4], os[4];
  void* out;
  int B, H, Sq, Sk, D;
  int mask_kind, causal;
  float scale;
};

// TPQ threads cooperate on one query; thread s of a query owns dims
// s, s+TPQ, s+2*TPQ, ... (interleaved so the TPQ threads hit distinct banks).
template <typename T, int TPQ>
__global__ void __launch_bounds__(kSdpaThreads) sdpa_kernel(const SdpaParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int QB = kSdpaThreads / TPQ;  // queries per CTA
  extern __shared__ float sm[];
  const int D = p.D;
  float* Ks = sm;                  // [BK][D]
  float* Vs = sm + kSdpaBK * D;    // [BK][D]
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * QB;
  const int tid = threadIdx.x;
  const int qi = tid / TPQ, sl = tid % TPQ;
  const int iq = q0 + qi;
  const bool qvalid = iq < p.Sq;
  const T* Q = static_cast<const T*>(p.q);
  const T* K = static_cast<const T*>(p.k);
  const T* V = static_cast<const T*>(p.v);
  const int nd = (D - sl + TPQ - 1) / TPQ;  // dims owned by this thread
  float qv[kSliceMax], o[kSliceMax];
#pragma unroll
  for (int i = 0; i < kSliceMax; ++i) {
    const int d = sl + TPQ * i;
    qv[i] = (qvalid && i < nd) ? to_f32<T>(Q[b * p.qs[0] + h * p.qs[1] + (long long)iq * p.qs[2] + d]) : 0.f;
    o[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  int kend = p.Sk;
  if (p.causal) kend = min(p.Sk, q0 + QB);
  for (int k0 = 0; k0 < kend; k0 += kSdpaBK) {
    __syncthreads();
    const int nk = min(kSdpaBK, kend - k0);
    for (int idx = tid; idx < kSdpaBK * D; idx += kSdpaThreads) {
      const int j = idx / D, d = idx % D;
      float kx = 0.f, vx = 0.f;
      if (j < nk) {
        kx = to_f32<T>(K[b * p.ks[0] + h * p.ks[1] + (long long)(k0 + j) * p.ks[2] + d]);
        vx = to_f32<T>(V[b * p.vs[0] + h * p.vs[1] + (long long)(k0 + j) * p.vs[2] + d]);
      }
      Ks[idx] = kx;
      Vs[idx] = vx;
    }
    __syncthreads();
    float s[kSdpaBK];
    float bmax = -INFINITY;
#pragma unroll 4
    for (int j = 0; j < kSdpaBK; ++j) {
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < kSliceMax; ++i)
        if (i < nd) d = fmaf(qv[i], Ks[j * D + sl + TPQ * i], d);
#pragma unroll
      for (int off = TPQ / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      float sc = d * p.scale;
      const int jk = k0 + j;
      bool keep = j < nk;
      if (keep && p.causal && jk > iq) keep = false;
      if (keep && p.mask_kind != 0) {
        const long long mo = b * p.ms[0] + h * p.ms[1] + (long long)iq * p.ms[2] + (long long)jk * p.ms[3];
        if (!qvalid) keep = false;
        else if (p.mask_kind == 1) keep = static_cast<const uint8_t*>(p.mask)[mo] != 0;
        else sc += to_f32<T>(static_cast<const T*>(p.mask)[mo]);
      }
      s[j] = keep ? sc : -INFINITY;
      bmax = fmaxf(bmax, s[j]);
    }
    const float m_new = fmaxf(m, bmax);
    if (m_new == -INFINITY) continue;  // everything so far masked
    const float alpha = expf(m - m_new);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < kSliceMax; ++i) o[i] *= alpha;
#pragma unroll 4
    for (int j = 0; j < kSdpaBK; ++j) {
      const float pr = expf(s[j] - m_new);
      l += pr;
#pragma unroll
      for (int i = 0; i < kSliceMax; ++i)
        if (i < nd) o[i] = fmaf(pr, Vs[j * D + sl + TPQ * i], o[i]);
    }
    m = m_new;
  }
  if (!qvalid) return;
  T* O = static_cast<T*>(p.out);
  const float inv = 1.0f / l;  // l == 0 (fully masked row) yields NaN, as the reference
#pragma unroll
  for (int i = 0; i < kSliceMax; ++i) {
    if (i < nd) {
      const int d = sl + TPQ * i;
      O[b * p.os[0] + h * p.os[1] + (long long)iq * p.os[2] + d] =
          from_f32<T>(l > 0.f ? o[i] * inv : NAN);
    }
  }
}

template <typename T>
static int launch_sdpa(const SdpaParams& p, cudaStream_t st) {
  int tpq = (p.D + kSliceMax - 1) / kSliceMax;
  int t2 = 1;
  while (t2 < tpq) t2 *= 2;
  const int qb = kSdpaThreads / t2;
  dim3 grid((unsigned)((p.Sq + qb - 1) / qb), (unsigned)(p.B * p.H));
  const size_t smem = (size_t)2 * kSdpaBK * p.D * sizeof(float);
  cudaError_t e;
  switch (t2) {
    case 1: e = cudaFuncSetAttribute(sdpa_kernel<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      launch_pdl(sdpa_kernel<T, 1>, dim3(grid), dim3(kSdpaThreads), smem, st, 1, p); break;
    case 2: e = cudaFuncSetAttribute(sdpa_kernel<T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      launch_pdl(sdpa_kernel<T, 2>, dim3(grid), dim3(kSdpaThreads), smem, st, 1, p); break;
    case 4: e = cudaFuncSetAttribute(sdpa_kernel<T, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      launch_pdl(sdpa_kernel<T, 4>, dim3(grid), dim3(kSdpaThreads), smem, st, 1, p); break;
    default: e = cudaFuncSetAttribute(sdpa_kernel<T, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      launch_pdl(sdpa_kernel<T, 8>, dim3(grid), dim3(kSdpaThreads), smem, st, 1, p); break;
  }
  if (e != cudaSuccess) return check_cuda(e, "sdpa attribute");
  count_launch();
  return check_cuda(cudaGetLastError(), "sdpa launch");
}

}  // namespace attn
}  // namespace fml

using namespace fml;

namespace fml {
int neb_prefill_tensor_core(const void* q, const int64_t qs[4], const void* k_pool, const void* v_pool,
                            const int32_t* slot_of, const int32_t* start_pos, void* out, int64_t B, int64_t T,
                            int64_t H, int64_t D, int64_t max_seq, int64_t slots, float scale, int dtype,
                            cudaStream_t st);
int sdpa_tensor_core(const void* q, const int64_t qs[4], const void* k, const int64_t ks[4], const void* v,
                     const int64_t vs[4], int mask_kind, int is_causal, float scale, void* out,
                     const int64_t os[4], int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int dtype,
                     cudaStream_t st);
}

extern "C" int neb_attention(const void* q, const int64_t q_strides[4], const void* k_pool,
                             const void* v_pool, const int32_t* slot_of, const int32_t* start_pos,
                             void* out, int64_t batch, int64_t t, int64_t heads, int64_t head_dim,
                             int64_t max_seq, int64_t pool_slots, float scale, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "neb_attention: bad dtype");
  if (!q || !q_strides || !k_pool || !v_pool || !slot_of || !start_pos || !out)
    return fail(FML_EINVAL, "neb_attention: null pointer");
  if (batch <= 0 || t <= 0 || heads <= 0 || head_dim <= 0 || max_seq <= 0 || pool_slots <= 0)
    return fail(FML_EINVAL, "neb_attention: sizes must be positive");
  if (head_dim > attn::kMaxD) return fail(FML_EUNSUPPORTED, "neb_attention: head_dim > 256");
  if (q_strides[3] != 1) return fail(FML_EUNSUPPORTED, "neb_attention: q innermost stride must be 1");
  if (batch * t * heads * 8 > (1ll << 31) - 1) return fail(FML_EUNSUPPORTED, "neb_attention: too many queries");
  // Key splits per query (combined in a cluster of at most 8): as many as
  // keep every CTA of the launch resident at once (two per SM: the bulk-copy
  // pipeline keeps 96 KB in flight per CTA), so each CTA streams a long run
  // of keys and no split spills into a second wave; measured on B200, more
  // and shorter CTAs lose to their per-CTA start-up.  Depends only on the
  // launch shape (not on the device-side positions), so a captured decode
  // step keeps a valid split.
  // Steps of several tokens per request (prefill) run on the tensor cores
  // when the layout allows (sdpa_tc.cu); single-token decode steps stream
  // the keys with the bulk-copy kernel below.
  if (t > 1) {
    const int rc = neb_prefill_tensor_core(q, q_strides, k_pool, v_pool, slot_of, start_pos, out, batch, t, heads,
                                           head_dim, max_seq, pool_slots, scale, dtype,
                                           reinterpret_cast<cudaStream_t>(stream));
    if (rc != FML_EUNSUPPORTED) return rc;
  }
  const long long nq = batch * t * heads;
  const long long target = 2LL * num_sms(current_device());
  int nsplit = (int)std::min<long long>(8, std::max<long long>(1, target / nq));
  nsplit = (int)std::min<long long>(nsplit, std::max<long long>(1, max_seq / 64));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FML_F32)
    return attn::dispatch_neb<float>(q, q_strides, k_pool, v_pool, slot_of, start_pos, out, batch,
                                     t, heads, head_dim, max_seq, scale, nsplit, st);
  if (dtype == FML_BF16)
    return attn::dispatch_neb<__nv_bfloat16>(q, q_strides, k_pool, v_pool, slot_of, start_pos, out,
                                             batch, t, heads, head_dim, max_seq, scale, nsplit, st);
  return attn::dispatch_neb<__half>(q, q_strides, k_pool, v_pool, slot_of, start_pos, out, batch, t,
                                    heads, head_dim, max_seq, scale, nsplit, st);
}

extern "C" int fml_sdpa(const void* q, const int64_t q_strides[4], const void* k,
                        const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                        const void* mask, const int64_t mask_strides[4], int mask_kind,
                        int is_causal, float scale, void* out, const int64_t out_strides[4],
                        int64_t batch, int64_t heads, int64_t sq, int64_t sk, int64_t d, int dtype,
                        void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "sdpa: bad dtype");
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return fail(FML_EINVAL, "sdpa: null pointer");
  if (batch <= 0 || heads <= 0 || sq <= 0 || sk <= 0 || d <= 0)
    return fail(FML_EINVAL, "sdpa: sizes must be positive");
  if (d > 256) return fail(FML_EUNSUPPORTED, "sdpa: head dim > 256");
  if (mask_kind < 0 || mask_kind > 2) return fail(FML_EINVAL, "sdpa: bad mask kind");
  if (mask_kind != 0 && (!mask || !mask_strides)) return fail(FML_EINVAL, "sdpa: mask pointer missing");
  if (mask_kind != 0 && is_causal) return fail(FML_EINVAL, "sdpa: attn_mask cannot be combined with is_causal");
  if (batch * heads > 65535) return fail(FML_EUNSUPPORTED, "sdpa: batch*heads > 65535");
  attn::SdpaParams p = {};
  p.q = q; p.k = k; p.v = v; p.mask = mask; p.out = out;
  for (int i = 0; i < 4; ++i) {
    p.qs[i] = q_strides[i]; p.ks[i] = k_strides[i]; p.vs[i] = v_strides[i];
    p.os[i] = out_strides[i]; p.ms[i] = mask_kind ? mask_strides[i] : 0;
  }
  p.B = (int)batch; p.H = (int)heads; p.Sq = (int)sq; p.Sk = (int)sk; p.D = (int)d;
  p.mask_kind = mask_kind; p.causal = is_causal ? 1 : 0; p.scale = scale;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // 16-bit attention without an explicit mask runs on the tensor cores
  // (sdpa_tc.cu); fp32 keeps the exact CUDA-core recurrence below.
  const int rc = sdpa_tensor_core(q, q_strides, k, k_strides, v, v_strides, mask_kind, is_causal, scale, out,
                                  out_strides, batch, heads, sq, sk, d, dtype, st);
  if (rc != FML_EUNSUPPORTED) return rc;
  if (dtype == FML_F32) return attn::launch_sdpa<float>(p, st);
  if (dtype == FML_BF16) return attn::launch_sdpa<__nv_bfloat16>(p, st);
  return attn::launch_sdpa<__half>(p, st);
}
