// tcgen05 GEMM with fused bias / GELU / residual epilogue for sm_100a.
//
// Replaces the Triton tile template of the reference
// (src/forgeml/_triton.py:6-62, launched by :65-93) and the cuBLAS F.linear
// calls of Nebula (src/nebula/runtime.py:131-133,145,152-153,186).
//
// Design (one persistent kernel, warp-specialised, 288 threads):
//   warps 5..8  TMA producers (P or Q operand x even or odd pipeline step):
//               2-D tiled loads of 128-byte K slabs into a ring of shared-
//               memory stages (SWIZZLE_128B), or one bulk copy per stage of
//               a pre-packed weight.  A stage's copies go out in one
//               instruction across lanes: a warp's copies otherwise complete
//               one after another.
//   warp 4      TMEM allocator + single-thread UMMA issuer
//               (tcgen05.mma, M=128 or a CTA pair's 256, N=BN, fp32
//               accumulate in TMEM, two accumulator buffers so the epilogue
//               of tile t overlaps the main loop of tile t+1); descriptors
//               are precomputed and stepped by constant offsets.
//   warps 0..3  epilogue (TMEM lane quadrant = warp): tcgen05.ld the
//               accumulator, apply the reference's rounding contract (round
//               to output dtype, + bias, round, GELU in fp32), optional
//               residual add, store.
//   warps 9..12 (wide 16-bit tiles only) epilogue helpers: the second half
//               of each tile's columns, so that two warps per TMEM lane
//               quadrant share a tile's epilogue.
//
// The kernel works in "MMA space": D[i][j] = sum_k P[i][k] * Q[j][k] where P
// supplies the 128 TMEM lanes and Q the BN columns.  For ordinary shapes
// P = A and Q = B^T; for skinny M ("swap") P = B^T and Q = A so that the wide
// weight dimension fills the 128-row tile and the small batch becomes the
// UMMA N dimension.  Each operand may be K-major or MN-major in global
// memory (both are native UMMA smem layouts), so row-major A, [K,N] weights
// (ForgeML) and [N,K] weights (Nebula) need no copies.
//
// Split-K: for few output tiles the K range is split across the CTAs of a
// thread-block cluster; each CTA pushes its partial rows to the row's owner
// CTA with st.async into distributed shared memory (no global scratch, no
// round trip).  Large 16-bit GEMMs run as CTA pairs (cta_group::2, 256-row
// tiles, each CTA loading half of Q).
#include <algorithm>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.cuh"
#include "peer_layout.cuh"

namespace fml {
namespace gemm {

constexpr int kBM = 128;        // UMMA M
constexpr int kSlab = 128;      // bytes of K per smem row (one swizzle row)
// Warp roles: 0-3 epilogue (TMEM lane quadrant = warp), 4 UMMA issuer,
// 5-8 TMA producers, 9-12 epilogue helpers (wide tiles, threads_of()).
constexpr int kMmaWarp = 4;
constexpr int kProducerWarp0 = 5;
constexpr int kThreads = 288;   // 9 warps
constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block
constexpr int kMaxStages = 8;
constexpr int kPromoteKb = 2;  // K slabs per promoted chunk (fp32 path)

struct Params {
  int I, J;              // rows of P and of Q (MMA space)
  int num_kb;            // K blocks of kSlab bytes over the (effective) reduction
  int slabs;             // K slabs carried by one pipeline stage (1, 2 or 4)
  int tiles_i, tiles_j, num_tiles, group_i;
  int ksplit;            // CTAs per cluster sharing one tile's K range
  int fmt;               // 0 f16, 1 bf16, 2 tf32
  int p_mn, q_mn;        // 1 if the operand is MN-major in smem
  int swap;              // 1: out[j][i], 0: out[i][j]
  int out_dtype;
  int act;
  int stages;
  int esize;             // element size of the MMA inputs (2 or 4)
  void* out;
  long long ldo;
  const void* bias;
  long long bias_stride;
  const void* residual;
  long long ldr;
  int rows_out, cols_out;  // M, N of the output
  int red_stride;          // floats per row of the split-K partial buffer
  int promote_kb;          // K slabs per TMEM chunk when partial sums are promoted to registers
  const uint8_t* p_packed; // P pre-packed as swizzled 16 KB tiles (nullptr: P comes through tmP)
  // Fused decode linear (FUSED kernels: pre-packed 16-bit weight, one tile per cluster).
  // LayerNorm over ln_k columns of x (the Q operand), by the epilogue warps:
  //   ln_mode 1 (prologue): Q = LN(x) written into the stages (no Q loads);
  //   ln_mode 2 (fold): Q = x through tmQ, P = W diag(gamma) packed, and the
  //     epilogue applies out = rstd * (acc - mean * fold_s[n]) + fold_c[n].
  int ln_mode;
  const float* fold_s;     // sum over k of the packed (gamma-scaled) weight row
  const float* fold_c;     // W . beta per feature (nullptr: zero)
  const void* ln_x;
  long long ln_ldx;
  const void* ln_g;
  const void* ln_b;
  float ln_eps;
  int ln_k;
  // KV-append epilogue: output feature n >= kv_q_cols goes to the K (then V) pool.
  void* kv_k;              // nullptr: no KV epilogue
  void* kv_v;
  const int32_t* kv_slot;
  const int32_t* kv_start;
  int kv_q_cols, kv_cols, kv_heads, kv_hd, kv_max_seq, kv_tq;
  // SUM all-reduce over the TP group (peer buffers) fused into the epilogue.
  int ar_on;
  peer::View ar;
};

struct Smem {
  uint32_t stage_base;  // 1024-aligned smem address of stage 0
  uint32_t stage_bytes;
  uint32_t p_bytes;
  uint32_t bars;        // base of the barrier block
  uint32_t red;         // split-K partial buffer
  uint32_t aux;         // FUSED kernels: LayerNorm statistics and all-reduce staging
};

__device__ __forceinline__ uint32_t bar_full(const Smem& s, int i) { return s.bars + 8 * i; }
__device__ __forceinline__ uint32_t bar_empty(const Smem& s, int i) {
  return s.bars + 8 * (kMaxStages + i);
}
__device__ __forceinline__ uint32_t bar_tfull(const Smem& s, int a) {
  return s.bars + 8 * (2 * kMaxStages + a);
}
__device__ __forceinline__ uint32_t bar_tempty(const Smem& s, int a) {
  return s.bars + 8 * (2 * kMaxStages + 2 + a);
}
// Split-K: completes once every other CTA of the cluster has pushed its
// partial rows of this CTA's output slice (transaction bytes of st.async).
__device__ __forceinline__ uint32_t bar_recv(const Smem& s) {
  return s.bars + 8 * (2 * kMaxStages + 4);
}
// CTA pair: each CTA tells the other it is done with TMEM before either frees it.
__device__ __forceinline__ uint32_t bar_dealloc(const Smem& s) {
  return s.bars + 8 * (2 * kMaxStages + 5);
}
__device__ __forceinline__ uint32_t bar_drain(const Smem& s) {
  return s.bars + 8 * (2 * kMaxStages + 6);
}
// LayerNorm prologue: completes once every other CTA of the cluster has
// pushed its row statistics of its K slice.
__device__ __forceinline__ uint32_t bar_ln(const Smem& s) {
  return s.bars + 8 * (2 * kMaxStages + 7);
}
constexpr int kNumBars = 2 * kMaxStages + 8;
constexpr int kBarBytes = 8 * kNumBars + 16;  // + tmem holder

// Wide tiles (BN >= 128, 16-bit, not fused) add four epilogue helper warps
// (warps 9-12, TMEM lane quadrant = warp % 4): without a split-K reduction
// a tile's columns are shared between the four epilogue warps (first half)
// and the helpers (second half).  One warp per quadrant and SM sub-partition
// leaves the epilogue latency-bound; at short K (a few dozen slabs) that
// epilogue, not the main loop, sets the tile rate.
constexpr int kHelperWarp0 = 9;
// Per epilogue warp (8 on wide tiles): a 32-row x 64-byte staging block and
// 64 bytes of bias (kEpiWarpBytes).
constexpr int kEpiStageBytes = 8 * (32 * 64 + 64);
template <int BN, bool PROMOTE, bool FUSED>
struct EpiHelp {
  static constexpr bool on = BN >= 128 && !PROMOTE && !FUSED;
};
template <int BN, bool PROMOTE, bool FUSED>
constexpr int threads_of() {
  return EpiHelp<BN, PROMOTE, FUSED>::on ? kThreads + 128 : kThreads;
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& ti, int& tj) {
  int per_group = p.group_i * p.tiles_j;
  int g = t / per_group;
  int first_i = g * p.group_i;
  int gsize = min(p.group_i, p.tiles_i - first_i);
  int local = t - g * per_group;
  ti = first_i + local % gsize;
  tj = local / gsize;
}

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
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
// Asynchronous store of 16 bytes into another CTA's shared memory; the
// bytes are reported as transactions on that CTA's mbarrier `mbar`.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float a, float b, float c, float d, uint32_t mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ void fence_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Epilogue, per output element (m, n) with fp32 accumulator v: the reference
// template's rounding contract (src/forgeml/_triton.py:43-57), round to the
// output dtype, add bias and round, apply GELU, then (Nebula's residual
// extension) round and add residual.  Callers loop over elements without
// unrolling (one inlined copy of the GELU code): unrolled copies per element
// overflow the instruction cache and stall every warp of the CTA.  The
// vectorised row path below is the exception, 32 elements in pairs.
// ---------------------------------------------------------------------------
// Epilogue for one output element at MMA coordinates (i, j) with fp32 value v.
__device__ __forceinline__ void epilogue_store(const Params& p, int i, int j, float v) {
  int m, n;
  if (p.swap) { m = j; n = i; } else { m = i; n = j; }
  if (m >= p.rows_out || n >= p.cols_out) return;
  const int od = p.out_dtype;
  float x = round_to(v, od);
  if (p.bias != nullptr) {
    float b;
    if (od == FML_F32) b = reinterpret_cast<const float*>(p.bias)[n * p.bias_stride];
    else if (od == FML_BF16) b = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.bias)[n * p.bias_stride]);
    else b = __half2float(reinterpret_cast<const __half*>(p.bias)[n * p.bias_stride]);
    x = round_to(x + b, od);
  }
  if (p.act == FML_ACT_GELU_ERF) x = gelu_erf(x);
  else if (p.act == FML_ACT_GELU_TANH) x = gelu_tanh(x);
  long long off = (long long)m * p.ldo + n;
  if (p.residual != nullptr) {
    long long roff = (long long)m * p.ldr + n;
    float r;
    if (od == FML_F32) r = reinterpret_cast<const float*>(p.residual)[roff];
    else if (od == FML_BF16) r = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.residual)[roff]);
    else r = __half2float(reinterpret_cast<const __half*>(p.residual)[roff]);
    x = round_to(x, od) + r;
  }
  if (od == FML_F32) reinterpret_cast<float*>(p.out)[off] = x;
  else if (od == FML_BF16) reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(x);
  else reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(x);
}

// Eight consecutive 16-bit bias values bias[n0 .. n0+7] as floats: one
// 16-byte load when the bias is contiguous and aligned there.
__device__ __forceinline__ void load_bias8(const Params& p, int n0, float (&bv)[8]) {
  const bool bf = p.out_dtype == FML_BF16;
  const uint16_t* bb = reinterpret_cast<const uint16_t*>(p.bias);
  auto cvt = [&](uint32_t h) {
    return bf ? __uint_as_float(h << 16) : __half2float(__ushort_as_half((unsigned short)h));
  };
  if (p.bias_stride == 1 && (reinterpret_cast<uintptr_t>(bb + n0) & 15) == 0) {
    const uint4 r = *reinterpret_cast<const uint4*>(bb + n0);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      bv[2 * i] = cvt(w[i] & 0xffffu);
      bv[2 * i + 1] = cvt(w[i] >> 16);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) bv[e] = cvt(bb[(long long)(n0 + e) * p.bias_stride]);
  }
}

// Fast path: 32 consecutive output columns of one row (non-swap), 16-bit
// output, no residual, aligned.  Applies the same per-element contract.
__device__ __forceinline__ bool epilogue_row32_fast(const Params& p, int m, int n0,
                                                    const float (&v)[32]) {
  if (p.swap || p.residual != nullptr || p.out_dtype == FML_F32) return false;
  if (m >= p.rows_out || n0 + 32 > p.cols_out) return false;
  long long off = (long long)m * p.ldo + n0;
  if ((off & 7) != 0 || (reinterpret_cast<uintptr_t>(p.out) & 15) != 0) return false;
  const int od = p.out_dtype;
  uint32_t packed[16];
  float bv[8];
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    if (p.bias != nullptr && (e & 7) == 0) load_bias8(p, n0 + e, bv);
    float x0 = round_to(v[e], od), x1 = round_to(v[e + 1], od);
    if (p.bias != nullptr) {
      x0 = round_to(x0 + bv[e & 7], od);
      x1 = round_to(x1 + bv[(e & 7) + 1], od);
    }
    if (p.act == FML_ACT_GELU_ERF) { x0 = gelu_erf(x0); x1 = gelu_erf(x1); }
    else if (p.act == FML_ACT_GELU_TANH) { x0 = gelu_tanh(x0); x1 = gelu_tanh(x1); }
    if (od == FML_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
      packed[e / 2] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(x0, x1);
      packed[e / 2] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + off);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  return true;
}

__device__ __forceinline__ float h2f(uint32_t v, bool bf) {
  return bf ? __uint_as_float((v & 0xffffu) << 16) : __half2float(__ushort_as_half((unsigned short)(v & 0xffffu)));
}
__device__ __forceinline__ uint32_t f2h(float v, bool bf) {
  return bf ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v))
            : (uint32_t)__half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ void unpack8(const uint4& r, bool bf, float (&v)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = h2f(w[i], bf);
    v[2 * i + 1] = h2f(w[i] >> 16, bf);
  }
}
// Epilogue value of output (m, n) from the fp32 accumulator v: the same
// contract as epilogue_store, without the store.
__device__ __forceinline__ float epilogue_value(const Params& p, int m, int n, float v) {
  const int od = p.out_dtype;
  float x = round_to(v, od);
  if (p.bias != nullptr) {
    float b;
    if (od == FML_F32) b = reinterpret_cast<const float*>(p.bias)[n * p.bias_stride];
    else if (od == FML_BF16) b = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.bias)[n * p.bias_stride]);
    else b = __half2float(reinterpret_cast<const __half*>(p.bias)[n * p.bias_stride]);
    x = round_to(x + b, od);
  }
  if (p.act == FML_ACT_GELU_ERF) x = gelu_erf(x);
  else if (p.act == FML_ACT_GELU_TANH) x = gelu_tanh(x);
  if (p.residual != nullptr) {
    const long long roff = (long long)m * p.ldr + n;
    float r;
    if (od == FML_F32) r = reinterpret_cast<const float*>(p.residual)[roff];
    else if (od == FML_BF16) r = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.residual)[roff]);
    else r = __half2float(reinterpret_cast<const __half*>(p.residual)[roff]);
    x = round_to(x, od) + r;
  }
  return x;
}

__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Sum of the split-K partials of eight outputs: element e of source CTA r at
// shared address red + r * src_stride + e * e_stride (bytes), added in
// source order.  All loads of one source are independent; the values stay in
// registers (compile-time indices only).
__device__ __forceinline__ void red_sum8(uint32_t red, int src_stride, int e_stride, int nsrc, float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
  for (int r = 0; r < nsrc; ++r) {
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = ld_shared_f32(red + (uint32_t)(r * src_stride + e * e_stride));
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] += t[e];
  }
}

__device__ __forceinline__ uint4 pack8_16(const float (&x)[8], bool bf) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (bf) {
      __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Eight consecutive outputs (m, n0..n0+7) with the epilogue contract of
// epilogue_store (from the split-K buffer, or from TMEM for tiles whose
// epilogue has a residual or an fp32 output).  Outputs with 16-byte aligned
// rows take a straight-line path: round, bias, GELU, residual (16-byte
// loads) and 16-byte stores; GELU runs in a rolled loop that rotates the
// eight registers (one copy of its code, nothing indexed dynamically, so
// nothing goes to local memory).  Other cases store element by element.
__device__ __forceinline__ void epilogue_store8(const Params& p, int m, int n0, float (&x)[8],
                                                const uint4* res_pre = nullptr) {
  if (m >= p.rows_out || n0 >= p.cols_out) return;
  const int od = p.out_dtype;
  const long long off = (long long)m * p.ldo + n0;
  const long long roff = (long long)m * p.ldr + n0;
  const long long ve = od == FML_F32 ? 4 : 8;  // elements per 16 bytes
  const bool vec = n0 + 8 <= p.cols_out && (off % ve) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                   (p.residual == nullptr ||
                    ((roff % ve) == 0 && (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0));
  if (!vec) {
#pragma unroll 1
    for (int e = 0; e < 8; ++e) {
      const float v = x[0];
#pragma unroll
      for (int i = 0; i < 7; ++i) x[i] = x[i + 1];
      if (n0 + e < p.cols_out) {
        const float y = epilogue_value(p, m, n0 + e, v);
        if (od == FML_F32) reinterpret_cast<float*>(p.out)[off + e] = y;
        else if (od == FML_BF16) reinterpret_cast<__nv_bfloat16*>(p.out)[off + e] = __float2bfloat16_rn(y);
        else reinterpret_cast<__half*>(p.out)[off + e] = __float2half_rn(y);
      }
    }
    return;
  }
  const bool bf = od == FML_BF16;
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = round_to(x[e], od);
  if (p.bias != nullptr) {
    if (od == FML_F32) {
      const float* bb = reinterpret_cast<const float*>(p.bias);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = x[e] + bb[(long long)(n0 + e) * p.bias_stride];
    } else {
      const uint16_t* bb = reinterpret_cast<const uint16_t*>(p.bias);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = round_to(x[e] + h2f(bb[(long long)(n0 + e) * p.bias_stride], bf), od);
    }
  }
  if (p.act != FML_ACT_NONE) {
    const bool erf_act = p.act == FML_ACT_GELU_ERF;
#pragma unroll 1
    for (int e = 0; e < 8; ++e) {
      const float g = erf_act ? gelu_erf(x[0]) : gelu_tanh(x[0]);
#pragma unroll
      for (int i = 0; i < 7; ++i) x[i] = x[i + 1];
      x[7] = g;
    }
  }
  if (od == FML_F32) {
    if (p.residual != nullptr) {
      const float4* rp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.residual) + roff);
      const float4 r0 = rp[0], r1 = rp[1];
      x[0] += r0.x; x[1] += r0.y; x[2] += r0.z; x[3] += r0.w;
      x[4] += r1.x; x[5] += r1.y; x[6] += r1.z; x[7] += r1.w;
    }
    float4* op = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off);
    op[0] = make_float4(x[0], x[1], x[2], x[3]);
    op[1] = make_float4(x[4], x[5], x[6], x[7]);
    return;
  }
  if (p.residual != nullptr) {
    const uint4 rv = res_pre != nullptr ? *res_pre
                                        : *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.residual) + roff);
    float r[8];
    unpack8(rv, bf, r);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = round_to(x[e], od) + r[e];
  }
  *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + off) = pack8_16(x, bf);
}

// ---------------------------------------------------------------------------
// Fused decode linear (FUSED kernels).  Nebula's decode step chains
//   LayerNorm -> QKV GEMM -> KV append            (src/nebula/runtime.py:130-138)
//   o GEMM -> SUM all-reduce -> + residual        (runtime.py:145-146)
//   LayerNorm -> up GEMM + GELU                   (runtime.py:151-152)
//   down GEMM -> SUM all-reduce -> + residual     (runtime.py:153-154)
// and the FUSED kernels run each line as one launch: the LayerNorm of the Q
// operand is computed by the epilogue warps while the weight stream starts
// (they are idle until the accumulator is ready), the KV rows go from the
// split-K reduction straight into the cache pools, and the row-parallel
// partial is exchanged with the other TP ranks over NVLink from the epilogue.
//
// Shared-memory block after the split-K buffer:
//   stats [8][BN] float2   each cluster CTA's row sums of its K slice
//   rowst [BN] float2      row mean and 1/sqrt(var + eps)
//   ep    [8] u32          exchange epochs of this CTA's sub-blocks
//   stage [128][32] u16    the rounded partial, feature-major, for the exchange
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int aux_rowst(int bn) { return 8 * bn * 8; }
__host__ __device__ constexpr int aux_ep(int bn) { return aux_rowst(bn) + bn * 8; }
__host__ __device__ constexpr int aux_stage(int bn) { return (aux_ep(bn) + 32 + 15) / 16 * 16; }
__host__ __device__ constexpr int aux_bytes(int bn) {
  return aux_stage(bn) + 128 * peer::kSubTokens * 2;
}

__device__ __forceinline__ void st_async_v2(uint32_t addr, float a, float b, uint32_t mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "f"(a), "f"(b), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void st_shared_v2(uint32_t addr, float a, float b) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ float2 ld_shared_v2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_u2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Barrier of the 128 epilogue threads that also ANDs a predicate over them,
// so that every thread takes the same branch afterwards.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)(v ? 1 : 0))
      : "memory");
  return r != 0;
}

// LayerNorm of the Q operand (x rows = tokens) into this CTA's pipeline
// stages, in the SWIZZLE_128B K-major image a TMA load would produce:
//   y = (x - mean) / sqrt(var + eps) * gamma + beta   over all ln_k columns,
// rounded to the 16-bit dtype (src/nebula/runtime.py:130,151; biased
// variance as F.layer_norm).  Each CTA of the split-K cluster reads only its
// K slice: it sums (x - x[r][0]) and its square over the slice, the cluster
// exchanges these partials through distributed shared memory, and every CTA
// adds them in cluster-rank order (identical statistics in every CTA).  The
// shift by the row's first element keeps var = E[d^2] - E[d]^2 well
// conditioned.  Then the slice is normalised stage by stage; each stage is
// handed to the UMMA warp like a TMA stage (one arrival on its full barrier).
// All 128 threads run every barrier; a timed-out wait only clears the result.
template <int BN>
__device__ bool ln_stats(const Params& p, const Smem& s, int ksplit, uint32_t crank, int kb_begin, int kb_end,
                         int tid) {
  constexpr int TPR = 128 / BN;  // threads per row
  const int r = tid / TPR, q = tid % TPR;
  const bool bf = p.fmt == 1;
  const bool valid = r < p.J;
  const uint16_t* xr = static_cast<const uint16_t*>(p.ln_x) + (long long)(valid ? r : 0) * p.ln_ldx;
  const int nchunk = (kb_end - kb_begin) * (kSlab / 16);
  const int e0 = kb_begin * (kSlab / 2);
  float shift = 0.f, s1 = 0.f, s2 = 0.f;
  if (valid) {
    shift = h2f(xr[0], bf);
#pragma unroll 4
    for (int c = q; c < nchunk; c += TPR) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + e0 + c * 8);
      float v[8];
      unpack8(raw, bf, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[e] - shift;
        s1 += d;
        s2 += d * d;
      }
    }
  }
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  const uint32_t stats = s.aux;
  const uint32_t rowst = s.aux + aux_rowst(BN);
  const uint32_t bar = bar_ln(s);
  if (ksplit > 1 && tid == 0) mbar_arrive_expect_tx(bar, (uint32_t)((ksplit - 1) * BN * 8));
  if (q == 0) {
    const uint32_t slot = stats + (uint32_t)(((int)crank * BN + r) * 8);
    st_shared_v2(slot, s1, s2);
    for (int c = 0; c < ksplit; ++c)
      if (c != (int)crank) st_async_v2(mapa(slot, (uint32_t)c), s1, s2, mapa(bar, (uint32_t)c));
  }
  bool ok = true;
  if (ksplit > 1) ok = mbar_wait_cluster(bar, 0, DEV_ERR_REDUCE_TIMEOUT);
  epi_bar_sync();
  if (q == 0) {
    float S1 = 0.f, S2 = 0.f;
    for (int c = 0; c < ksplit; ++c) {
      const float2 v = ld_shared_v2(stats + (uint32_t)((c * BN + r) * 8));
      S1 += v.x;
      S2 += v.y;
    }
    const float kf = (float)p.ln_k;
    const float md = S1 / kf;
    const float var = fmaxf(S2 / kf - md * md, 0.f);
    st_shared_v2(rowst + r * 8, shift + md, 1.0f / sqrtf(var + p.ln_eps));
  }
  epi_bar_sync();
  return ok;
}

template <int BN>
__device__ bool ln_prologue(const Params& p, const Smem& s, int ksplit, uint32_t crank, int kb_begin,
                            int kb_end, int tid) {
  constexpr int TPR = 128 / BN;  // threads per row
  const int r = tid / TPR, q = tid % TPR;
  const bool bf = p.fmt == 1;
  const bool valid = r < p.J;
  const uint16_t* xr = static_cast<const uint16_t*>(p.ln_x) + (long long)(valid ? r : 0) * p.ln_ldx;
  bool ok = ln_stats<BN>(p, s, ksplit, crank, kb_begin, kb_end, tid);
  const float2 ms = ld_shared_v2(s.aux + aux_rowst(BN) + r * 8);
  const uint16_t* g = static_cast<const uint16_t*>(p.ln_g);
  const uint16_t* b = static_cast<const uint16_t*>(p.ln_b);
  int stage = 0;
  uint32_t phase = 0;
  for (int kb = kb_begin; kb < kb_end; ++kb) {
    // first pass over the ring: the stage is free; later: wait for the UMMA
    // warp to release it (as a TMA producer would)
    if (!mbar_wait(bar_empty(s, stage), phase ^ 1u, DEV_ERR_GEMM_TIMEOUT)) ok = false;
    const uint32_t qb = s.stage_base + stage * s.stage_bytes + s.p_bytes;
    const int kel = kb * (kSlab / 2);
#pragma unroll
    for (int c = q; c < kSlab / 16; c += TPR) {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (valid) {
        float v[8], gv[8], bv[8];
        unpack8(*reinterpret_cast<const uint4*>(xr + kel + c * 8), bf, v);
        unpack8(*reinterpret_cast<const uint4*>(g + kel + c * 8), bf, gv);
        unpack8(*reinterpret_cast<const uint4*>(b + kel + c * 8), bf, bv);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float t0 = (v[e] - ms.x) * ms.y, t1 = (v[e + 1] - ms.x) * ms.y;
          t0 = t0 * gv[e] + bv[e];
          t1 = t1 * gv[e + 1] + bv[e + 1];
          w[e / 2] = f2h(t0, bf) | (f2h(t1, bf) << 16);
        }
      }
      st_shared_u4(qb + (uint32_t)(r * kSlab + ((c ^ (r & 7)) << 4)), w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
    epi_bar_sync();
    if (tid == 0) mbar_arrive(bar_full(s, stage));
    if (++stage == p.stages) { stage = 0; phase ^= 1u; }
  }
  return ok;
}

// KV-append epilogue: output features n >= kv_q_cols of token m go to
// pool[slot_of[b], head, start_pos[b] + t, d] of the K or V pool
// (m = b * tq + t), rounded to the 16-bit dtype like the GEMM output they
// replace (src/nebula/cache.py:161-165 via runtime.py:136-138); a position
// out of range raises DEV_ERR_ATTN_RANGE like neb_kv_append.
// Eight consecutive features n0..n0+7 of token m (one head, same K or V
// pool: q_cols and head_dim are multiples of 8) as one 16-byte store.
__device__ __forceinline__ void kv_store8(const Params& p, int n0, int m, const float (&x)[8]) {
  if (n0 >= p.cols_out || m >= p.J) return;
  const int nn = n0 - p.kv_q_cols;
  const bool is_v = nn >= p.kv_cols;
  const int c = is_v ? nn - p.kv_cols : nn;
  const int head = c / p.kv_hd, d = c - head * p.kv_hd;
  const int b = m / p.kv_tq, t = m - b * p.kv_tq;
  const int slot = p.kv_slot[b];
  const int pos = p.kv_start[b] + t;
  if (slot < 0 || pos < 0 || pos >= p.kv_max_seq) {
    raise_device_error(DEV_ERR_ATTN_RANGE);
    return;
  }
  const long long dst = (((long long)slot * p.kv_heads + head) * p.kv_max_seq + pos) * p.kv_hd + d;
  uint16_t* pool = static_cast<uint16_t*>(is_v ? p.kv_v : p.kv_k);
  *reinterpret_cast<uint4*>(pool + dst) = pack8_16(x, p.fmt == 1);
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"((unsigned short)v) : "memory");
}

// LayerNorm folded into the product (ln_mode 2): with P = W diag(gamma),
//   LN(x) W^T = rstd * (x P^T - mean * sum_k P[n][k]) + W beta
// for eight consecutive features n0.. of token row r of this tile; the row's
// mean and rstd come from ln_stats.  (The reference rounds LN(x) to the model
// dtype before the product; here the product sees it unrounded.)
__device__ __forceinline__ void ln_fold8(const Params& p, const Smem& s, int BNv, int r, int n0, float (&x)[8]) {
  const float2 ms = ld_shared_v2(s.aux + (uint32_t)aux_rowst(BNv) + (uint32_t)(r * 8));
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int n = min(n0 + e, p.cols_out - 1);
    const float c = p.fold_c != nullptr ? p.fold_c[n] : 0.f;
    x[e] = ms.y * (x[e] - ms.x * p.fold_s[n]) + c;
  }
}

// The global inputs of one reduction item (output row m, features n0..n0+7):
// the LayerNorm-fold vectors and the residual row segment, loaded before the
// accumulator is ready so that their latency is off the epilogue's path.
struct ItemInputs {
  float fs[8], fc[8];
  uint4 res;
};
__device__ __forceinline__ void item_prefetch(const Params& p, int m, int n0, ItemInputs& in) {
  if (p.ln_mode == 2) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int n = min(n0 + e, p.cols_out - 1);
      in.fs[e] = p.fold_s[n];
      in.fc[e] = p.fold_c != nullptr ? p.fold_c[n] : 0.f;
    }
  }
  if (p.residual != nullptr && p.out_dtype != FML_F32 && m < p.rows_out && n0 + 8 <= p.cols_out) {
    const long long roff = (long long)m * p.ldr + n0;
    if ((roff & 7) == 0 && (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0)
      in.res = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.residual) + roff);
  }
}
__device__ __forceinline__ void ln_fold8_pre(const Params& p, const Smem& s, int BNv, int r, const ItemInputs& in,
                                             float (&x)[8]) {
  const float2 ms = ld_shared_v2(s.aux + (uint32_t)aux_rowst(BNv) + (uint32_t)(r * 8));
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = ms.y * (x[e] - ms.x * in.fs[e]) + in.fc[e];
}

// All-reduce epilogue of one owner CTA: its rows_per features (rows r0.. of
// tile ti) x 32 tokens, already rounded into the staging block.  Per 16-
// feature sub-block c: push the 1 KB block into slot `rank` of every rank's
// buffer (NVLink stores), fence, raise flag [rank][c] on every peer with the
// sub-block's epoch, wait for every peer's flag [q][c], then
//   out = round(round(sum over q in rank order of slot q) + residual)
// (ParallelContext.all_reduce + `x + part`, src/nebula/parallel.py:112-116,
// runtime.py:146,154), identical on every rank.  Epochs and the two buffer
// sets follow the standalone all-reduce's protocol (allreduce.cu) with the
// sub-block as the unit.  Waits are bounded (DEV_ERR_AR_TIMEOUT).
template <int BN>
__device__ bool ar_exchange(const Params& p, const Smem& s, int ti, int r0, int rows_per, int tid) {
  const peer::View& a = p.ar;
  const int W = a.lay.world, rank = a.rank;
  const bool bf = p.fmt == 1;
  const int nsb = rows_per / peer::kSubFeatures;
  const int c0 = (ti * kBM + r0) / peer::kSubFeatures;
  const int nsub_valid = (p.cols_out + peer::kSubFeatures - 1) / peer::kSubFeatures;
  constexpr int kSubBytes = peer::kSubFeatures * peer::kSubTokens * 2;  // 1 KB
  constexpr int kChunks = kSubBytes / 16;
  const uint32_t ep = s.aux + aux_ep(BN);
  const uint32_t stg = s.aux + aux_stage(BN);
  uint32_t* epochs = reinterpret_cast<uint32_t*>(a.base[rank] + a.lay.ex_epoch_off(0));
  if (tid < nsb) st_shared_u32(ep + 4 * tid, c0 + tid < nsub_valid ? epochs[c0 + tid] + 1u : 0u);
  epi_bar_sync();  // staging block and epochs visible to all epilogue threads
  for (int u = tid; u < nsb * W * kChunks; u += 128) {
    const int sb = u / (W * kChunks), rem = u - sb * (W * kChunks);
    const int q = rem / kChunks, ch = rem - q * kChunks;
    if (c0 + sb >= nsub_valid) continue;
    const uint32_t e = ld_shared_u32(ep + 4 * sb);
    const uint4 v = ld_shared_u4(stg + (uint32_t)(sb * kSubBytes + ch * 16));
    *reinterpret_cast<uint4*>(a.base[q] + a.lay.ex_data_off((int)(e & 1u), rank) + (long long)(c0 + sb) * kSubBytes +
                              ch * 16) = v;
  }
  __threadfence_system();
  epi_bar_sync();
  for (int u = tid; u < nsb * W; u += 128) {
    const int sb = u / W, q = u - sb * W;
    if (q == rank || c0 + sb >= nsub_valid) continue;
    const uint32_t e = ld_shared_u32(ep + 4 * sb);
    peer::st_release_sys(reinterpret_cast<uint32_t*>(a.base[q] + a.lay.ex_flag_off((int)(e & 1u), rank, c0 + sb)), e);
  }
  bool got = true;
  for (int u = tid; u < nsb * W; u += 128) {
    const int sb = u / W, q = u - sb * W;
    if (q == rank || c0 + sb >= nsub_valid) continue;
    const uint32_t e = ld_shared_u32(ep + 4 * sb);
    const uint32_t* f = reinterpret_cast<const uint32_t*>(a.base[rank] + a.lay.ex_flag_off((int)(e & 1u), q, c0 + sb));
    const long long t0 = clock64();
    while (peer::ld_acquire_sys(f) != e) {
      if (clock64() - t0 > a.timeout_cycles) {
        raise_device_error(DEV_ERR_AR_TIMEOUT);
        got = false;
        break;
      }
    }
  }
  got = epi_bar_and(got);  // every peer's block of this CTA's sub-blocks has landed
  const uint16_t* res = static_cast<const uint16_t*>(p.residual);
  uint16_t* out = static_cast<uint16_t*>(p.out);
  for (int u = tid; u < rows_per * p.J; u += 128) {
    const int f = u % rows_per, m = u / rows_per;
    const int sb = f / peer::kSubFeatures;
    const int n = ti * kBM + r0 + f;
    if (n >= p.cols_out) continue;
    const uint32_t e = ld_shared_u32(ep + 4 * sb);
    const long long off = (long long)(c0 + sb) * kSubBytes + ((f % peer::kSubFeatures) * peer::kSubTokens + m) * 2;
    float acc = 0.f;
    for (int q = 0; q < W; ++q)
      acc += h2f(*reinterpret_cast<const uint16_t*>(a.base[rank] + a.lay.ex_data_off((int)(e & 1u), q) + off), bf);
    float x = h2f(f2h(acc, bf), bf);  // the all-reduced partial in the model dtype
    if (res != nullptr) x = x + h2f(res[(long long)m * p.ldr + n], bf);
    out[(long long)m * p.ldo + n] = (uint16_t)f2h(x, bf);
  }
  epi_bar_sync();
  if (tid < nsb && c0 + tid < nsub_valid) epochs[c0 + tid] = ld_shared_u32(ep + 4 * tid);
  return got;
}

// Narrow tiles are register-bounded for two CTAs per SM (the decode weight
// stream, ~100 KB of shared memory each).
// PAIR: a CTA pair (cluster of 2) computes 256 x BN tiles with cta_group::2
// UMMAs; each CTA loads its 128 rows of P and BN/2 rows of Q (16-bit,
// non-split only).
// FUSED: the decode linear with the LayerNorm prologue, KV-append and
// all-reduce epilogues (pre-packed 16-bit P, swapped, one tile per cluster,
// always through the split-K reduction buffer).
// One warp's 32 rows x 32 columns of a wide 16-bit tile (thread = row, v =
// its 32 accumulators, output columns n0..n0+31 of rows m0..m0+31), stored
// coalesced: the rows are staged in this warp's block of shared memory
// (16-byte chunk q of row r at r*64 + (q ^ ((r >> 1) & 3))*16, conflict-free
// both ways) and written back by the warp 8 rows x 64 bytes per instruction,
// so the L2 sees whole sectors instead of 16-byte pieces of 32 rows.  The
// block's bias (64 bytes) and residual rows are loaded one block ahead
// (stage_prefetch) so that their latency overlaps the previous block.
// Epilogue contract of epilogue_store.
constexpr int kEpiWarpBytes = 32 * 64 + 64;  // staged rows + the block's bias

struct StageIn {
  uint4 bias;    // lanes 0-3: 16 bytes each of bias[n0 .. n0+31]
  uint4 res[4];  // residual rows cr + 8*it, 16-byte chunk cq
};

// Whether the block at (m0, n0) can take the staged path (warp-uniform).
__device__ __forceinline__ bool stage_ok(const Params& p, int m0, int n0) {
  return m0 + 32 <= p.rows_out && n0 + 32 <= p.cols_out && (p.ldo & 7) == 0 &&
         (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
         (p.bias == nullptr || (p.bias_stride == 1 && ((reinterpret_cast<uintptr_t>(p.bias) + 2 * n0) & 15) == 0)) &&
         (p.residual == nullptr || ((p.ldr & 7) == 0 && (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0));
}

__device__ __forceinline__ void stage_prefetch(const Params& p, int m0, int n0, int lane, StageIn& in) {
  if (p.bias != nullptr && lane < 4)
    in.bias = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.bias) + n0 + lane * 8);
  if (p.residual != nullptr) {
    const uint16_t* rb = reinterpret_cast<const uint16_t*>(p.residual);
#pragma unroll
    for (int it = 0; it < 4; ++it)
      in.res[it] = *reinterpret_cast<const uint4*>(rb + (long long)(m0 + (lane >> 2) + 8 * it) * p.ldr + n0 +
                                                   (lane & 3) * 8);
  }
}

__device__ __forceinline__ void stage_store32(const Params& p, uint32_t stg, int m0, int n0, int lane,
                                              const float (&v)[32], const StageIn& in) {
  const int od = p.out_dtype;
  const bool bf = od == FML_BF16;
  const int cr = lane >> 2, cq = lane & 3;  // coalesced pass: row within 8, 16-byte chunk
  auto slot = [&](int r, int q) { return stg + (uint32_t)(r * 64 + ((q ^ ((r >> 1) & 3)) * 16)); };
  const uint32_t bslot = stg + 32 * 64;
  if (p.bias != nullptr && lane < 4) st_shared_u4(bslot + lane * 16, in.bias.x, in.bias.y, in.bias.z, in.bias.w);
  if (p.residual != nullptr) {
#pragma unroll
    for (int it = 0; it < 4; ++it) st_shared_u4(slot(cr + 8 * it, cq), in.res[it].x, in.res[it].y, in.res[it].z, in.res[it].w);
  }
  __syncwarp();
  // One copy of the per-8-column code (a rolled loop; the 32 values rotate
  // by 8 registers per pass, nothing is indexed dynamically): the epilogue
  // runs beside the producer and MMA warps' code on each SM sub-partition,
  // and a small instruction footprint keeps it out of instruction misses.
  float w[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) w[e] = v[e];
#pragma unroll 1
  for (int q = 0; q < 4; ++q) {
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = round_to(w[e], od);
#pragma unroll
    for (int e = 0; e < 24; ++e) w[e] = w[e + 8];
    if (p.bias != nullptr) {
      float bv[8];
      unpack8(ld_shared_u4(bslot + q * 16), bf, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = round_to(x[e] + bv[e], od);
    }
    if (p.act != FML_ACT_NONE) {
      const bool erf_act = p.act == FML_ACT_GELU_ERF;
#pragma unroll 1
      for (int e = 0; e < 8; ++e) {  // one copy of the GELU code, registers rotated
        const float g = erf_act ? gelu_erf(x[0]) : gelu_tanh(x[0]);
#pragma unroll
        for (int k = 0; k < 7; ++k) x[k] = x[k + 1];
        x[7] = g;
      }
    }
    if (p.residual != nullptr) {
      float r[8];
      unpack8(ld_shared_u4(slot(lane, q)), bf, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = round_to(x[e], od) + r[e];
    }
    const uint4 o = pack8_16(x, bf);
    st_shared_u4(slot(lane, q), o.x, o.y, o.z, o.w);
  }
  __syncwarp();
  uint16_t* ob = reinterpret_cast<uint16_t*>(p.out);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = cr + 8 * it;
    *reinterpret_cast<uint4*>(ob + (long long)(m0 + r) * p.ldo + n0 + cq * 8) = ld_shared_u4(slot(r, cq));
  }
  __syncwarp();  // the block is refilled by the next one
}

template <int BN, bool PROMOTE, bool PAIR = false, bool FUSED = false>
__global__ void __launch_bounds__(threads_of<BN, PROMOTE, FUSED>(), (BN <= 64 && !PROMOTE) ? 2 : 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  Smem s;
  s.stage_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int S = p.slabs;
  s.p_bytes = S * kBM * kSlab;
  constexpr int kQRows = PAIR ? BN / 2 : BN;  // Q rows this CTA loads per tile
  constexpr int kTileM = PAIR ? 2 * kBM : kBM;  // output rows per tile
  s.stage_bytes = S * (kBM + kQRows) * kSlab;
  s.bars = s.stage_base + p.stages * s.stage_bytes;
  s.red = s.bars + kBarBytes;
  s.red = (s.red + 15u) & ~15u;
  s.aux = s.red + (uint32_t)(kBM * p.red_stride * 4 + 16);  // FUSED only (the split-K buffer is always there)
  const uint32_t tmem_holder = s.bars + 8 * kNumBars;

  const int ksplit = PAIR ? 1 : p.ksplit;
  constexpr bool kClusterLaunch = true;  // (ksplit > 1 or PAIR) -> launched as clusters
  const int csize = PAIR ? 2 : ksplit;
  const uint32_t crank = csize > 1 ? cluster_ctarank() : 0u;
  const bool leader = !PAIR || crank == 0;
  const int prank = PAIR ? (int)crank : 0;  // this CTA's half of a pair tile
  const int cluster_id = blockIdx.x / csize;
  const int num_clusters = gridDim.x / csize;
  const int kb_begin = PAIR ? 0 : (int)((long long)crank * p.num_kb / ksplit);
  const int kb_end = PAIR ? p.num_kb : (int)((long long)(crank + 1) * p.num_kb / ksplit);
  (void)kClusterLaunch;
  constexpr bool kHelp = EpiHelp<BN, PROMOTE, FUSED>::on;
  const bool help_on = kHelp && ksplit == 1;  // split-K tiles reduce through the 4-warp path

  constexpr int kAccStride = BN < 32 ? 32 : BN;
  constexpr int kTmemCols = (2 * kAccStride <= 32) ? 32
                            : (2 * kAccStride <= 64) ? 64
                            : (2 * kAccStride <= 128) ? 128
                            : (2 * kAccStride <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(bar_full(s, i), 2);  // one arrive from the P producer, one from the Q producer
      mbar_init(bar_empty(s, i), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull(s, a), 1);
      // a pair's leader hears both CTAs' epilogues (and helpers)
      mbar_init(bar_tempty(s, a), (PAIR ? 8 : 4) * (help_on ? 2 : 1));
    }
    mbar_init(bar_recv(s), 1);
    mbar_init(bar_ln(s), 1);
    mbar_init(bar_dealloc(s), 1);
    mbar_init(bar_drain(s), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == kMmaWarp) {
    if (PAIR) {
      tmem_alloc_pair(tmem_holder, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (csize > 1) cluster_sync_all();
  tc_fence_after();
  uint32_t tmem_base;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem_base) : "r"(tmem_holder) : "memory");

  const int bke = kSlab / p.esize;            // K elements per slab
  const int mn_box = kSlab / p.esize;         // MN elements per MN-major box
  const uint32_t slab_box_bytes = (uint32_t)bke * kSlab;  // bytes of one MN-major box

  if (warp >= kProducerWarp0 && warp < kHelperWarp0) {
    // ------------------------------------------------------------ producers
    // Four warps: P or Q operand x even or odd pipeline steps.  A warp's
    // bulk/TMA copies are processed one after another (about a memory
    // latency each), while copies issued by different warps, or by several
    // lanes of one instruction, are in flight together.  So every copy of
    // a stage's operand (one per slab, or per box for MN-major operands)
    // goes out in a single instruction across lanes, and consecutive steps
    // alternate between two warps.  Lane 0 waits for the free stage and arms
    // the full barrier with this operand's bytes.
    const int pw = warp - kProducerWarp0;
    const bool is_q = pw >= 2;
    const int parity = pw & 1;
    const CUtensorMap* tm = is_q ? &tmQ : &tmP;
    const int mn = is_q ? p.q_mn : p.p_mn;
    const int rows = is_q ? kQRows : kBM;
    const uint32_t op_off = is_q ? s.p_bytes : 0u;
    const uint32_t slab_bytes = (uint32_t)rows * kSlab;
    const bool packed = !is_q && p.p_packed != nullptr;
    // FUSED with the LayerNorm prologue: the epilogue warps write Q.
    const bool idle = FUSED && is_q && p.ln_mode == 1;
    const int nbox = mn ? rows / mn_box : 1;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool ok = true;
    // Constant (pre-packed) weights do not depend on the previous kernel:
    // start streaming the first tile's weight slabs into the free stages
    // before waiting for the previous grid (programmatic dependent launch).
    const int steps_first = cluster_id < p.num_tiles ? (kb_end - kb_begin + S - 1) / S : 0;
    const int pre_limit = packed ? min(p.stages, steps_first) : 0;
    if (pre_limit > 0 && lane == 0) {
      int ti0, tj0;
      tile_coords(p, cluster_id, ti0, tj0);
      for (int st = parity; st < pre_limit; st += 2) {
        const int kb = kb_begin + st * S;
        const int nsl = min(S, kb_end - kb);
        const uint32_t fb = bar_full(s, st);
        mbar_arrive_expect_tx(fb, (uint32_t)nsl * slab_bytes);
        bulk_load(s.stage_base + st * s.stage_bytes,
                  p.p_packed + ((size_t)ti0 * p.num_kb + kb) * (size_t)(kBM * kSlab), (uint32_t)nsl * slab_bytes, fb);
        issued_mask |= 1u << st;
      }
    }
    __syncwarp();
    pdl_wait();
    pdl_trigger();
    int step = 0;
    for (int t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
      int ti, tj;
      tile_coords(p, t, ti, tj);
      const int rbase = is_q ? tj * BN + prank * kQRows : ti * kTileM + prank * kBM;
      for (int kb = kb_begin; kb < kb_end; kb += S, ++step) {
        if (!idle && (step & 1) == parity && step >= pre_limit) {
          const int nsl = min(S, kb_end - kb);
          // A pair's copies all complete on the leader's full barrier, which
          // the leader's producer arms with both CTAs' bytes.
          const uint32_t fb = PAIR ? mapa(bar_full(s, stage), 0) : bar_full(s, stage);
          bool got = true;
          if (lane == 0) {
            got = mbar_wait(bar_empty(s, stage), phase ^ 1u, DEV_ERR_GEMM_TIMEOUT);
            if (got && leader) mbar_arrive_expect_tx(bar_full(s, stage), (uint32_t)nsl * slab_bytes * (PAIR ? 2u : 1u));
          }
          if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) { ok = false; break; }
          const uint32_t dst0 = s.stage_base + stage * s.stage_bytes + op_off;
          if (packed) {
            // The tile's slabs are stored pre-swizzled and consecutive.
            if (lane == 0)
              bulk_load(dst0, p.p_packed + ((size_t)ti * p.num_kb + kb) * (size_t)(kBM * kSlab),
                        (uint32_t)nsl * slab_bytes, fb);
          } else if (lane < nsl * nbox) {
            const int sl = lane / nbox, b = lane % nbox;
            const uint32_t dst = dst0 + sl * slab_bytes + b * slab_box_bytes;
            const int x = mn ? rbase + b * mn_box : (kb + sl) * bke;
            const int y = mn ? (kb + sl) * bke : rbase;
            if (PAIR) tma_load_2d_pair(tm, fb, dst, x, y);
            else tma_load_2d(tm, fb, dst, x, y);
          }
          __syncwarp();
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        }
        if (++stage == p.stages) { stage = 0; phase ^= 1u; }
      }
    }
    if (!ok && lane == 0) {
      // Unwind: let every load we issued land before the CTA can exit.
      for (int i = 0; i < p.stages; ++i)
        if (issued_mask & (1u << i))
          mbar_wait(bar_full(s, i), (issued_parity >> i) & 1u, DEV_ERR_GEMM_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ UMMA issuer
    pdl_wait();
    pdl_trigger();
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc(p.fmt, p.p_mn, p.q_mn, BN, PAIR ? 256 : 128);
      const uint32_t p_lbo = p.p_mn ? slab_box_bytes : 16u;
      const uint32_t q_lbo = p.q_mn ? slab_box_bytes : 16u;
      // Descriptors of stage 0 / slab 0 / K step 0; everything else is a
      // constant offset added to the start-address field (address >> 4).
      // Per UMMA K step (32 bytes of K): within the swizzle row for K-major,
      // (32/esize) rows of 128 B for MN-major.
      const uint64_t dp0 = umma_desc_sw128(s.stage_base, p_lbo, 1024u);
      const uint64_t dq0 = umma_desc_sw128(s.stage_base + s.p_bytes, q_lbo, 1024u);
      const uint32_t d_stage = s.stage_bytes >> 4;
      const uint32_t dp_slab = (kBM * kSlab) >> 4, dq_slab = (kQRows * kSlab) >> 4;
      const uint32_t dp_k = (p.p_mn ? (uint32_t)(32 / p.esize) * kSlab : 32u) >> 4;
      const uint32_t dq_k = (p.q_mn ? (uint32_t)(32 / p.esize) * kSlab : 32u) >> 4;
      const bool tf32 = p.fmt == 2;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
        // PROMOTE (fp32 / 3xTF32): the K range is cut into chunks of
        // promote_kb slabs, each accumulated from zero in TMEM and summed by
        // the epilogue in fp32 registers with round-to-nearest adds, which
        // bounds the tensor core accumulator's rounding error.
        int kb = kb_begin;
        while (kb < kb_end && ok) {
          const int kb_stop = PROMOTE ? min(kb + p.promote_kb, kb_end) : kb_end;
          if (!mbar_wait(bar_tempty(s, acc), acc_phase ^ 1u, DEV_ERR_GEMM_TIMEOUT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * kAccStride;
          uint32_t accum = 0u;
          for (; kb < kb_stop; kb += S) {
            if (!mbar_wait(bar_full(s, stage), phase, DEV_ERR_GEMM_TIMEOUT)) { ok = false; break; }
            tc_fence_after();
            const int nsl = min(S, kb_end - kb);
            const uint64_t dp = dp0 + stage * d_stage, dq = dq0 + stage * d_stage;
            for (int sl = 0; sl < nsl; ++sl) {
              const uint64_t ap = dp + sl * dp_slab, bq = dq + sl * dq_slab;
              if (PAIR) {
#pragma unroll
                for (int k = 0; k < 4; ++k) { umma_f16_pair(d_tmem, ap + k * dp_k, bq + k * dq_k, idesc, accum); accum = 1u; }
              } else if (tf32) {
#pragma unroll
                for (int k = 0; k < 4; ++k) { umma_tf32(d_tmem, ap + k * dp_k, bq + k * dq_k, idesc, accum); accum = 1u; }
              } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) { umma_f16(d_tmem, ap + k * dp_k, bq + k * dq_k, idesc, accum); accum = 1u; }
              }
            }
            if (PAIR) {
              umma_commit_pair(bar_empty(s, stage));
              umma_commit_pair(mapa(bar_empty(s, stage), 1));
            } else {
              umma_commit(bar_empty(s, stage));
            }
            if (++stage == p.stages) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          if (PAIR) {
            umma_commit_pair(bar_tfull(s, acc));
            umma_commit_pair(mapa(bar_tfull(s, acc), 1));
          } else {
            umma_commit(bar_tfull(s, acc));
          }
          if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
      }
      // Drain: every UMMA issued above has completed before TMEM is freed.
      if (PAIR) umma_commit_pair(bar_drain(s));
      else umma_commit(bar_drain(s));
      mbar_wait(bar_drain(s), 0, DEV_ERR_GEMM_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // bias / residual / output may belong to the previous grid
    pdl_trigger();
    const bool helper = kHelp && warp >= kHelperWarp0;
    const bool idle = helper && !help_on;
    const int quad = warp & 3;              // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;       // MMA row within the tile
    const int ep_tid = threadIdx.x;         // 0..127 (helpers: 288..415, no shared-buffer work)
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    constexpr int kChunks = (BN + 31) / 32;
    const int c_begin = helper ? kChunks / 2 : 0;               // this warp's 32-column chunks
    const int c_end = (help_on && !helper) ? kChunks / 2 : kChunks;
    float* red = reinterpret_cast<float*>(smem_raw + (s.red - smem_u32(smem_raw)));
    // Split-K (one tile per cluster): rows [crank*rows_per, +rows_per) of the
    // tile are owned by this CTA.  Every CTA pushes its partial of each row
    // to the row's owner (st.async into recv[src][row], own rows with plain
    // stores), so the owner needs no round trip: it waits on bar_recv for the
    // other CTAs' bytes and sums the ksplit partials of its slice.
    const int rows_per = kBM / ksplit;
    const int owner = row / rows_per, orow = row % rows_per;
    const uint32_t push_local = s.red + (uint32_t)(((crank * rows_per + orow) * p.red_stride) * 4);
    const uint32_t push_dst = (ksplit > 1 && owner != (int)crank) ? mapa(push_local, owner) : push_local;
    const uint32_t push_bar = ksplit > 1 ? mapa(bar_recv(s), owner) : 0u;
    auto push4 = [&](int col, float a, float b, float c, float d) {
      if (owner == (int)crank) st_shared_v4(push_local + col * 4, a, b, c, d);
      else st_async_v4(push_dst + col * 4, a, b, c, d, push_bar);
    };
    // FUSED kernels always reduce through the split-K buffer (also with one
    // CTA per tile), where the KV and all-reduce epilogues take over.
    // Narrow swapped tiles (the decode linears) also store through it: eight
    // outputs per thread as one vector instead of 32 scattered 2-byte stores.
    constexpr bool kRedAlways = FUSED;
    const bool use_red = ksplit > 1 || kRedAlways || (BN <= 32 && p.swap);
    if constexpr (FUSED) {
      if (p.ln_mode == 1 && cluster_id < p.num_tiles)
        ok = epi_bar_and(ln_prologue<BN>(p, s, ksplit, crank, kb_begin, kb_end, ep_tid));
      // fold: the statistics are computed while the main loop runs
      if (p.ln_mode == 2 && cluster_id < p.num_tiles)
        ok = epi_bar_and(ln_stats<BN>(p, s, ksplit, crank, kb_begin, kb_end, ep_tid));
    }
    for (int t = cluster_id; t < p.num_tiles && ok && !idle; t += num_clusters) {
      int ti, tj;
      tile_coords(p, t, ti, tj);
      const int i = ti * kTileM + prank * kBM + row;
      if (ksplit > 1 && ep_tid == 0)
        mbar_arrive_expect_tx(bar_recv(s), (uint32_t)((ksplit - 1) * rows_per * BN * 4));
      // swapped reduction tiles (the decode linears): this thread's first
      // item's global inputs, fetched while the main loop still runs
      ItemInputs pre;
      const bool have_pre = use_red && p.swap && ep_tid < (rows_per / 8) * BN;
      if (have_pre)
        item_prefetch(p, tj * BN + ep_tid % BN, ti * kBM + crank * rows_per + (ep_tid / BN) * 8, pre);
      float racc[PROMOTE ? BN : 1];
#pragma unroll
      for (int e = 0; e < (PROMOTE ? BN : 1); ++e) racc[e] = 0.f;
      const int nchunks = PROMOTE ? (kb_end - kb_begin + p.promote_kb - 1) / p.promote_kb : 1;
      // wide tiles: this warp's 32 x 32 blocks go through its staging slot;
      // the first block's bias / residual are fetched before the tile's
      // accumulator is ready
      const uint32_t stg = s.red + (uint32_t)((helper ? warp - kHelperWarp0 + 4 : warp) * kEpiWarpBytes);
      const bool staged = kHelp && help_on && !p.swap && p.out_dtype != FML_F32 &&
                          stage_ok(p, i - lane, tj * BN + c_begin * 32) &&
                          stage_ok(p, i - lane, tj * BN + (c_end - 1) * 32);
      StageIn pf;
      if (staged) stage_prefetch(p, i - lane, tj * BN + c_begin * 32, lane, pf);
      for (int ch = 0; ch < nchunks && ok; ++ch) {
        if (!mbar_wait(bar_tfull(s, acc), acc_phase, DEV_ERR_GEMM_TIMEOUT)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * kAccStride;
        if (PROMOTE) {
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e < BN) racc[(c * 32 + e) % (PROMOTE ? BN : 1)] += v[e];
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR && !leader) mbar_arrive_remote(mapa(bar_tempty(s, acc), 0));
            else mbar_arrive(bar_tempty(s, acc));
          }
        } else {
#pragma unroll 1
          for (int c = c_begin; c < c_end; ++c) {
            float v[32];
            tmem_ld32(tbase + c * 32, v);
            if (c == c_end - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
            if (PAIR && !leader) mbar_arrive_remote(mapa(bar_tempty(s, acc), 0));
            else mbar_arrive(bar_tempty(s, acc));
          }
            }
            const int nvalid = min(32, BN - c * 32);
            if (!use_red) {
              const int j0 = tj * BN + c * 32;
              if (staged) {
                const StageIn cur = pf;
                if (c + 1 < c_end) stage_prefetch(p, i - lane, j0 + 32, lane, pf);
                stage_store32(p, stg, i - lane, j0, lane, v, cur);
                continue;
              }
              if (nvalid == 32 && epilogue_row32_fast(p, i, j0, v)) continue;
              if (!p.swap) {
                // residual or fp32 output: 16-byte vectors of eight columns
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  if (8 * q < nvalid) {
                    float x[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[e] = v[8 * q + e];
                    epilogue_store8(p, i, j0 + 8 * q, x);
                  }
                }
              } else {
                // swapped: MMA row i is an output column, the 32 values are
                // 32 output rows; a rolled loop that rotates the registers
#pragma unroll 1
                for (int e = 0; e < nvalid; ++e) {
                  const float v0 = v[0];
#pragma unroll
                  for (int k = 0; k < 31; ++k) v[k] = v[k + 1];
                  epilogue_store(p, i, j0 + e, v0);
                }
              }
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                if (4 * q < nvalid) push4(c * 32 + 4 * q, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
          }
        }
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) break;
      if (PROMOTE) {
        if (!use_red && !p.swap) {
          // a row of BN consecutive output columns: 16-byte vectors of eight
#pragma unroll
          for (int q = 0; q < BN / 8; ++q) {
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = racc[8 * q + e];
            epilogue_store8(p, i, tj * BN + 8 * q, x);
          }
        } else if (!use_red) {
          // swapped: one output column, BN rows; a rolled loop that rotates
          // the registers (nothing indexed dynamically, no local memory)
#pragma unroll 1
          for (int e = 0; e < BN; ++e) {
            const float v0 = racc[0];
#pragma unroll
            for (int k = 0; k < BN - 1; ++k) racc[k] = racc[k + 1];
            epilogue_store(p, i, tj * BN + e, v0);
          }
        } else {
#pragma unroll
          for (int q = 0; q < BN / 4; ++q)
            push4(4 * q, racc[4 * q], racc[4 * q + 1], racc[4 * q + 2], racc[4 * q + 3]);
        }
      }
      if (use_red) {
        epi_bar_sync();  // own rows' plain stores visible to every epilogue thread
        if (FUSED) {
          // every thread must leave together: the exchange below has barriers
          const bool got = ksplit == 1 || mbar_wait_cluster(bar_recv(s), 0, DEV_ERR_REDUCE_TIMEOUT);
          if (!epi_bar_and(got)) { ok = false; break; }
        } else if (ksplit > 1 && !mbar_wait_cluster(bar_recv(s), 0, DEV_ERR_REDUCE_TIMEOUT)) {
          ok = false;
          break;
        }
        const int r0 = crank * rows_per;
        // Items of eight consecutive output columns of one output row.  swap:
        // output row = token (MMA column c), columns = features (MMA rows
        // rr0..rr0+7), consecutive threads on consecutive tokens (conflict-
        // free reads of the buffer); otherwise one MMA row, eight columns.
        const int src_stride = rows_per * p.red_stride * 4;  // bytes between source CTAs' slices
        const int row_bytes = p.red_stride * 4;
        const int items = p.swap ? (rows_per / 8) * BN : rows_per * (BN / 8);
        for (int idx = ep_tid; idx < items; idx += 128) {
          int rr0, c0;
          if (p.swap) { c0 = idx % BN; rr0 = (idx / BN) * 8; }
          else { rr0 = idx / (BN / 8); c0 = (idx % (BN / 8)) * 8; }
          const uint32_t base = s.red + (uint32_t)((rr0 * p.red_stride + c0) * 4);
          if constexpr (FUSED) {
            const int n0 = ti * kBM + r0 + rr0;  // first feature (the fused kernels are swapped)
            const int m = tj * BN + c0;
            float x[8];
            red_sum8(base, src_stride, row_bytes, ksplit, x);
            if (p.ln_mode == 2) {
              if (have_pre && idx == ep_tid) ln_fold8_pre(p, s, BN, c0, pre, x);
              else ln_fold8(p, s, BN, c0, n0, x);
            }
            if (p.ar_on) {
              // rounded partial -> staging block [feature][token] for the exchange
              const bool bf = p.fmt == 1;
#pragma unroll
              for (int e = 0; e < 8; ++e)
                st_shared_u16(s.aux + aux_stage(BN) + (uint32_t)(((rr0 + e) * peer::kSubTokens + c0) * 2), f2h(x[e], bf));
              continue;
            }
            if (p.kv_k != nullptr && n0 >= p.kv_q_cols) {
              kv_store8(p, n0, m, x);
              continue;
            }
            epilogue_store8(p, m, n0, x);
            continue;
          }
          float x[8];
          red_sum8(base, src_stride, p.swap ? row_bytes : 4, ksplit, x);
          if (p.swap) epilogue_store8(p, tj * BN + c0, ti * kBM + r0 + rr0, x,
                                      have_pre && idx == ep_tid && p.residual != nullptr ? &pre.res : nullptr);
          else epilogue_store8(p, ti * kBM + r0 + rr0, tj * BN + c0, x);
        }
        if (ksplit == 1) epi_bar_sync();  // the buffer is refilled by this CTA's next tile
        if constexpr (FUSED) {
          if (p.ar_on && !ar_exchange<BN>(p, s, ti, r0, rows_per, ep_tid)) ok = false;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    if (PAIR) {
      // Both CTAs are done with the pair's TMEM before either frees it.
      if (lane == 0) {
        const uint32_t peer = crank ^ 1u;
        if (leader) {
          mbar_wait_cluster(bar_dealloc(s), 0, DEV_ERR_GEMM_TIMEOUT);
          mbar_arrive_remote(mapa(bar_dealloc(s), peer));
        } else {
          mbar_arrive_remote(mapa(bar_dealloc(s), peer));
          mbar_wait_cluster(bar_dealloc(s), 0, DEV_ERR_GEMM_TIMEOUT);
        }
      }
      __syncwarp();
      tmem_dealloc_pair(tmem_base, kTmemCols);
    } else {
      tmem_dealloc(tmem_base, kTmemCols);
    }
  }
}

// ---------------------------------------------------------------------------
// Operand packing (workspace): K-major copy with 16-byte aligned rows, and the
// 3xTF32 split of fp32 operands.
//   mode 0: dst[r, k] = X[r, k]                              (width Kp)
//   mode 1: dst = [lo | hi | hi] (P side)                    (width 3 Kp)
//   mode 2: dst = [hi | lo | hi] (Q side)                    (width 3 Kp)
// so that P' . Q'^T = lo_P hi_Q + hi_P lo_Q + hi_P hi_Q, the three-product
// tf32 error-compensated form ("3xTF32"), smallest terms accumulated first.
// hi = x rounded to tf32 (cvt.rna), lo = x - hi rounded to tf32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

template <typename T>
__global__ void pack_kernel(const T* __restrict__ x, long long s_r, long long s_k, int R, int K,
                            int Kp, int mode, T* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  const int r0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
  const bool r_contig = (s_r == 1 && s_k != 1);
  // Load a 32x32 tile with the unit-stride dimension across threadIdx.x.
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    int r, k;
    if (r_contig) { r = r0 + threadIdx.x; k = k0 + yy; }
    else { r = r0 + yy; k = k0 + threadIdx.x; }
    float v = 0.f;
    if (r < R && k < K) v = to_f32<T>(x[(long long)r * s_r + (long long)k * s_k]);
    if (r_contig) tile[threadIdx.x][yy] = v;
    else tile[yy][threadIdx.x] = v;
  }
  __syncthreads();
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    const int r = r0 + yy, k = k0 + threadIdx.x;
    if (r >= R || k >= Kp) continue;
    const float v = tile[yy][threadIdx.x];  // zero in the padding columns
    if (mode == 0) {
      dst[(long long)r * Kp + k] = from_f32<T>(v);
    } else {
      const float hi = tf32_round(v);
      const float lo = tf32_round(v - hi);
      float* d = reinterpret_cast<float*>(dst) + (long long)r * 3 * Kp;
      if (mode == 1) { d[k] = lo; d[Kp + k] = hi; d[2 * Kp + k] = hi; }
      else { d[k] = hi; d[Kp + k] = lo; d[2 * Kp + k] = hi; }
    }
  }
}

// Constant-weight packing: W [N, K] (K contiguous, nn.Linear layout) becomes
// tiles of 128 rows x one 128-byte K slab, each stored exactly as the
// SWIZZLE_128B K-major shared-memory image the UMMA descriptor expects
// (16-byte chunk c of row r at r*128 + (c ^ (r & 7))*16), tiles of one
// 128-row band consecutive along K.  A decode-step GEMM then streams each
// weight band as one sequential run of 16 KB bulk copies.  Out-of-range rows
// and columns are zero.
template <typename T>
__global__ void pack_weight_kernel(const T* __restrict__ w, long long ldw, int n, int k, int num_kb,
                                   long long total_chunks, uint8_t* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = 16 / sizeof(T);  // elements per 16-byte chunk
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total_chunks;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx & 7);
    const int r = (int)((idx >> 3) & 127);
    const long long tile = idx >> 10;          // ti * num_kb + kb
    const int kb = (int)(tile % num_kb);
    const long long ti = tile / num_kb;
    const long long row = ti * kBM + r;
    const long long col = (long long)kb * (kSlab / sizeof(T)) + c * E;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < n) {
      const T* src = w + row * ldw + col;
      if (col + E <= k && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        T* e = reinterpret_cast<T*>(&v);
        for (int i = 0; i < E; ++i) e[i] = (col + i < k) ? src[i] : from_f32<T>(0.f);
      }
    }
    *reinterpret_cast<uint4*>(dst + tile * (kBM * kSlab) + r * kSlab + ((c ^ (r & 7)) * 16)) = v;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Operand description in MMA space: X[r][k] at ptr + r*s_r + k*s_k.
struct Operand {
  const void* ptr;
  long long s_r, s_k;
  long long rows, k;
  bool mn;       // MN-major (s_r == 1) when used directly
  bool pack;     // needs a packed copy in workspace
  size_t ws_off; // workspace offset of the packed copy
  long long kp;  // padded row length of the packed copy (elements)
  const void* pre = nullptr;  // caller-packed 3xTF32 image (fml_gemm_packed_b), read directly
};

// 3xTF32 split layout of one operand (pack_kernel modes): the A operand is
// stored [lo | hi | hi] and the B operand [hi | lo | hi] along K, so the
// product over the tripled K is A_lo B_hi + A_hi B_lo + A_hi B_hi whichever
// operand the plan puts in the 128-row (P) position.
static inline int split_mode(bool is_b, int dtype) { return dtype == FML_F32 ? (is_b ? 2 : 1) : 0; }

static inline long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }

// Decide whether TMA can address the operand directly.
static void classify(Operand& o, int dtype, int box_mn, bool allow_mn) {
  const long long es = (long long)dtype_size(dtype);
  o.pack = true;
  o.mn = false;
  if (dtype == FML_F32) return;  // 3xTF32 always splits into workspace
  if (reinterpret_cast<uintptr_t>(o.ptr) % 16 != 0) return;
  const bool k_unit = (o.s_k == 1 || o.k == 1);
  const bool r_unit = (o.s_r == 1 || o.rows == 1);
  if (k_unit) {
    long long stride_bytes = (o.rows == 1 ? round_up(o.k * es, 16) : o.s_r * es);
    if (stride_bytes % 16 == 0 && stride_bytes > 0 && (o.rows == 1 || o.s_r >= o.k)) {
      if (o.rows == 1) o.s_r = stride_bytes / es;
      if (o.k == 1) o.s_k = 1;
      o.pack = false;
      return;
    }
  }
  if (r_unit && allow_mn && box_mn % (128 / es) == 0) {
    long long stride_bytes = (o.k == 1 ? round_up(o.rows * es, 16) : o.s_k * es);
    if (stride_bytes % 16 == 0 && stride_bytes > 0 && (o.k == 1 || o.s_k >= o.rows)) {
      if (o.k == 1) o.s_k = stride_bytes / es;
      o.s_r = 1;
      o.mn = true;
      o.pack = false;
    }
  }
}

static int encode(CUtensorMap* map, const void* ptr, int dtype, bool tf32, bool mn,
                  long long rows, long long keff, long long stride_elems, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(FML_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const long long es = (long long)dtype_size(dtype);
  CUtensorMapDataType dt = dtype == FML_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == FML_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  (void)tf32;
  cuuint64_t dims[2], strides[1];
  cuuint32_t box[2], estr[2] = {1, 1};
  const cuuint32_t slab_elems = (cuuint32_t)(kSlab / es);
  if (!mn) {
    dims[0] = (cuuint64_t)keff;
    dims[1] = (cuuint64_t)rows;
    box[0] = slab_elems;
    box[1] = (cuuint32_t)box_rows;
  } else {
    dims[0] = (cuuint64_t)rows;
    dims[1] = (cuuint64_t)keff;
    box[0] = slab_elems;
    box[1] = slab_elems;  // one slab of K rows per box (kSlab/es)
  }
  strides[0] = (cuuint64_t)(stride_elems * es);
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FML_EINVAL, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) +
                                ") rows=" + std::to_string(rows) + " k=" + std::to_string(keff) +
                                " stride=" + std::to_string(stride_elems));
  return FML_OK;
}

struct Plan {
  bool pair = false;  // CTA-pair (cta_group::2) 256 x 256 tiles
  bool swap;
  bool promote;  // fp32: sum TMEM partials in fp32 registers every kPromoteKb slabs
  bool packed;   // P is a pre-packed constant weight (fml_linear_packed)
  bool fused = false;  // FUSED decode-linear kernel (neb_linear_fused)
  int bn;
  int ksplit;
  int stages;
  int slabs;     // K slabs per pipeline stage
  Operand P, Q;
  long long keff;  // effective reduction length (3*Kp for tf32)
  size_t ws_bytes;
};

static const int kBNs[] = {16, 32, 64, 128, 256};

static int smem_bytes_for(int bn, int stages, int ksplit, int* red_stride, int slabs = 1, bool pair = false,
                          bool fused = false) {
  int stage_bytes = slabs * (kBM + (pair ? bn / 2 : bn)) * kSlab;
  int rs = bn + 4;
  if (red_stride) *red_stride = rs;
  int red = (ksplit > 1 || fused || bn <= 32) ? kBM * rs * 4 + 16 : 0;  // narrow swapped tiles store through it
  // wide tiles without split-K stage their output rows for coalesced stores
  // (in the place of the unused split-K buffer)
  if (red == 0 && bn >= 128 && !fused) red = kEpiStageBytes;
  return 1024 + stages * stage_bytes + kBarBytes + 16 + red + (fused ? aux_bytes(bn) : 0);
}

// CTAs of one SM this configuration fits: shared memory, registers, threads
// and TMEM columns.  Computed here because the occupancy API reports one CTA
// per SM for any kernel that uses tcgen05, while the hardware co-schedules
// several when their resources fit (measured on B200).
template <int BN, bool PROMOTE>
static int per_sm_ctas(int smem) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, gemm_kernel<BN, PROMOTE>) != cudaSuccess) return 1;
  int dev = current_device(), smem_sm = 0;
  if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess || smem_sm <= 0)
    smem_sm = 233472;
  constexpr int threads = threads_of<BN, PROMOTE, false>();
  const int warps = threads / 32;
  const int regs_block = warps * ((fa.numRegs * 32 + 255) / 256) * 256;
  constexpr int acc = BN < 32 ? 32 : BN;
  constexpr int tmem_cols = (2 * acc <= 32) ? 32 : (2 * acc <= 64) ? 64 : (2 * acc <= 128) ? 128 : (2 * acc <= 256) ? 256 : 512;
  int n = smem_sm / (smem + (int)fa.sharedSizeBytes + 1024);
  n = std::min(n, 65536 / std::max(regs_block, 1));
  n = std::min(n, 2048 / threads);
  n = std::min(n, 512 / tmem_cols);
  return std::max(n, 1);
}

template <int BN, bool PROMOTE>
static int resident_ctas_t(int ksplit, int smem, int sms) {
  cudaFuncSetAttribute(gemm_kernel<BN, PROMOTE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  const int per_sm = per_sm_ctas<BN, PROMOTE>(smem);
  if (ksplit <= 1) return per_sm * sms;
  // Clusters: the occupancy API's count (one CTA per SM, whole clusters
  // inside a GPC) scaled by the CTAs an SM really holds.
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(ksplit);
  lc.blockDim = dim3(threads_of<BN, PROMOTE, false>());
  lc.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ksplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN, PROMOTE>, &lc) != cudaSuccess || n <= 0) return 0;
  return n * ksplit * per_sm;
}

// CTAs of this kernel configuration that can be resident at once (cached).
static int resident_ctas(int bn, bool promote, int ksplit, int smem, int sms) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int>, int> cache;
  const int dev = current_device();
  const auto key = std::make_tuple(dev, bn, promote ? 1 : 0, ksplit, smem, sms);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int r = 0;
  if (promote) {
    switch (bn) {
      case 16: r = resident_ctas_t<16, true>(ksplit, smem, sms); break;
      case 32: r = resident_ctas_t<32, true>(ksplit, smem, sms); break;
      case 64: r = resident_ctas_t<64, true>(ksplit, smem, sms); break;
    }
  } else {
    switch (bn) {
      case 16: r = resident_ctas_t<16, false>(ksplit, smem, sms); break;
      case 32: r = resident_ctas_t<32, false>(ksplit, smem, sms); break;
      case 64: r = resident_ctas_t<64, false>(ksplit, smem, sms); break;
      case 128: r = resident_ctas_t<128, false>(ksplit, smem, sms); break;
      case 256: r = resident_ctas_t<256, false>(ksplit, smem, sms); break;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = r;
  return r;
}

// Pipeline stages: the hint, else as many as fit; a pre-packed (decode)
// weight stream defaults to four one-slab stages, which keeps the CTA near
// 100 KB of shared memory so that the next kernel's CTAs are resident beside
// it and prefetch their weights during programmatic dependent launch.
static int stages_for(int bn, int ksplit, const fml_tile_cfg* cfg, int slabs, bool packed = false, bool pair = false) {
  int stages = packed ? 4 : kMaxStages;
  // The stage hint applies to single-CTA tiles; a CTA pair always takes the
  // deepest ring that fits (its stages are a third smaller).
  if (cfg && cfg->num_stages > 0 && !pair) stages = std::min(cfg->num_stages, kMaxStages);
  while (stages > 2 && smem_bytes_for(bn, stages, ksplit, nullptr, slabs, pair) > kSmemLimit) --stages;
  return stages;
}

// K slabs per stage: block_k elements of K per stage when hinted; by default
// four slabs (64 KB of weights per stage) for the bandwidth-bound narrow tiles
// (BN <= 64) streamed through TMA, one slab for pre-packed weights and for
// the wide compute-bound tiles.
static int slabs_for(const fml_tile_cfg* cfg, int dtype, bool promote, int bn, bool packed = false) {
  if (promote) return 1;
  if (!cfg || cfg->block_k <= 0) return (bn <= 64 && !packed) ? 4 : 1;
  const int s = cfg->block_k * (int)dtype_size(dtype) / kSlab;
  return s >= 4 ? 4 : (s >= 2 ? 2 : 1);
}

// Split-K and pipeline depth.  Each candidate split is costed by the rounds of
// co-resident CTAs it needs times the K slabs each CTA streams, plus a fixed
// per-tile cost and the cluster reduction; a split whose clusters cannot all
// be resident at once pays for the extra round.
static void choose_split(Plan& pl, long long tiles, long long num_kb, const fml_tile_cfg* cfg, int sms) {
  int best_ks = 1;
  double best_cost = 1e30;
  for (int ks : {1, 2, 4, 8}) {
    if (ks > 1 && (pl.bn > 128 || num_kb < 2LL * ks || tiles * 2 > sms)) continue;
    const int st = stages_for(pl.bn, ks, cfg, pl.slabs, pl.packed);
    const int smem = smem_bytes_for(pl.bn, st, ks, nullptr, pl.slabs, false, pl.fused);
    if (smem > kSmemLimit) continue;
    const int res = resident_ctas(pl.bn, pl.promote, ks, smem, sms);
    if (res <= 0) continue;
    const long long ctas = tiles * ks;
    const long long rounds = (ctas + res - 1) / res;
    const double per_cta = (double)((num_kb + ks - 1) / ks) + 6.0;
    const double cost = rounds * per_cta + (ks > 1 ? 4.0 : 0.0);
    if (cost < best_cost - 1e-9) { best_cost = cost; best_ks = ks; }
  }
  pl.ksplit = best_ks;
  pl.stages = stages_for(pl.bn, best_ks, cfg, pl.slabs, pl.packed);
}

static int pick_bn(const Plan& pl, long long I, long long J, const fml_tile_cfg* cfg, int sms) {
  int bn = 256;
  if (cfg && cfg->block_n > 0) {
    bn = 0;
    for (int c : kBNs)
      if (c >= std::min<long long>(cfg->block_n, 256)) { bn = c; break; }
    if (bn == 0) bn = 256;
  } else if (pl.swap) {
    bn = 256;
    for (int c : kBNs)
      if (c >= J) { bn = c; break; }
  } else {
    // Pick the wider tile unless it leaves too many SMs idle.
    long long ti = (I + kBM - 1) / kBM;
    auto util = [&](int c) {
      long long tiles = ti * ((J + c - 1) / c);
      long long waves = (tiles + sms - 1) / sms;
      return (double)tiles / (double)(waves * sms) * std::min(1.0, (double)J / c);
    };
    bn = 256;
    if (J <= 128) { for (int c : kBNs) if (c >= J) { bn = c; break; } }
    else if (util(128) > util(256) * 1.15) bn = 128;
  }
  if (pl.promote && bn > 64) bn = 64;  // register-resident row accumulator
  return bn;
}

static int make_plan(Plan& pl, const void* a, long long lda_m, long long lda_k, const void* b,
                     long long ldb_k, long long ldb_n, long long M, long long N, long long K,
                     int dtype, const fml_tile_cfg* cfg, int sms, const void* b_pre = nullptr) {
  pl.packed = false;
  pl.swap = (M <= 128 && N > M);
  if (pl.swap) {
    pl.P = Operand{b, ldb_n, ldb_k, N, K, false, false, 0, 0};
    pl.Q = Operand{a, lda_m, lda_k, M, K, false, false, 0, 0};
  } else {
    pl.P = Operand{a, lda_m, lda_k, M, K, false, false, 0, 0};
    pl.Q = Operand{b, ldb_n, ldb_k, N, K, false, false, 0, 0};
  }
  const long long J = pl.Q.rows, I = pl.P.rows;
  pl.promote = (dtype == FML_F32);
  pl.bn = pick_bn(pl, I, J, cfg, sms);
  classify(pl.P, dtype, kBM, true);
  classify(pl.Q, dtype, pl.bn, true);
  const long long es = (long long)dtype_size(dtype);
  const long long kp = round_up(K, 16 / es);
  pl.keff = dtype == FML_F32 ? 3 * kp : K;
  if (b_pre) {  // fp32 B already split by fml_gemm_pack_b
    Operand& bo = pl.swap ? pl.P : pl.Q;
    bo.pack = false;
    bo.mn = false;
    bo.pre = b_pre;
    bo.kp = kp;
  }
  size_t ws = 0;
  for (Operand* o : {&pl.P, &pl.Q}) {
    if (!o->pack) continue;
    o->kp = kp;
    o->ws_off = ws;
    ws += (size_t)round_up(o->rows * (dtype == FML_F32 ? 3 * kp : kp) * es, 256);
  }
  pl.ws_bytes = ws;
  const long long tiles = ((I + kBM - 1) / kBM) * ((J + pl.bn - 1) / pl.bn);
  const long long num_kb = (pl.keff * es + kSlab - 1) / kSlab;
  pl.slabs = slabs_for(cfg, dtype, pl.promote, pl.bn);
  // CTA pairs (256 x 256 per pair, each CTA loading half of Q) when the tile
  // hint asks for 256-row tiles (block_m = 256).  By default wide tiles run
  // on single CTAs: measured on B200, a stage lands about every 1000 cycles
  // in both forms whatever its bytes, and single 128 x 256 tiles with the
  // eight-warp staged epilogue were 2-20 % faster than pairs on every shape
  // of configs 2 and 3 (8192^3, 4096 x 768 x 3072, 4096 x 2304 x 768).
  pl.pair = cfg && cfg->block_m == 256 && !pl.swap && !pl.promote && dtype != FML_F32 && pl.bn == 256 &&
            I >= 2 * kBM && pl.slabs == 1;
  if (pl.pair) {
    pl.ksplit = 1;
    pl.stages = stages_for(pl.bn, 1, cfg, pl.slabs, false, true);
  } else {
    choose_split(pl, tiles, num_kb, cfg, sms);
  }
  if (smem_bytes_for(pl.bn, pl.stages, pl.ksplit, nullptr, pl.slabs, pl.pair) > kSmemLimit)
    return fail(FML_EUNSUPPORTED, "gemm tile does not fit in shared memory");
  return FML_OK;
}

template <int BN, bool PROMOTE, bool PAIR = false, bool FUSED = false>
static int launch_bn(const CUtensorMap& mp, const CUtensorMap& mq, const Params& prm, int grid,
                     int smem, cudaStream_t st) {
  static std::once_flag once[64];
  const int dev = current_device();
  cudaError_t e = cudaSuccess;
  std::call_once(once[dev & 63], [&]() {
    e = cudaFuncSetAttribute(gemm_kernel<BN, PROMOTE, PAIR, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemLimit);
  });
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemm)");
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(threads_of<BN, PROMOTE, FUSED>());
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++na;
  if (prm.ksplit > 1 || PAIR) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = PAIR ? 2 : prm.ksplit;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  lc.attrs = attr;
  lc.numAttrs = na;
  e = cudaLaunchKernelEx(&lc, gemm_kernel<BN, PROMOTE, PAIR, FUSED>, mp, mq, prm);
  if (e != cudaSuccess) return check_cuda(e, "gemm launch");
  count_launch();
  return FML_OK;
}

// Fill the kernel parameters shared by every entry point and launch.
static int launch_plan(const Plan& pl, const CUtensorMap& mp, const CUtensorMap& mq, int dtype, int act,
                       const void* bias, long long bias_stride, const void* residual, long long ldr, void* c,
                       long long ldc, long long m, long long n, const uint8_t* p_packed, int sms,
                       cudaStream_t st, const Params* fusion = nullptr) {
  Params prm = fusion ? *fusion : Params{};
  prm.I = (int)pl.P.rows;
  prm.J = (int)pl.Q.rows;
  const long long es = (long long)dtype_size(dtype);
  prm.num_kb = (int)((pl.keff * es + kSlab - 1) / kSlab);
  prm.slabs = pl.slabs;
  prm.tiles_i = (int)((prm.I + (pl.pair ? 2 : 1) * kBM - 1) / ((pl.pair ? 2 : 1) * kBM));
  prm.tiles_j = (int)((prm.J + pl.bn - 1) / pl.bn);
  prm.num_tiles = prm.tiles_i * prm.tiles_j;
  // Tile raster: groups of group_i tile rows advance along N together
  // (measured on B200: 8 for CTA pairs, 16 for single CTAs).
  prm.group_i = std::min(prm.tiles_i, pl.pair ? 8 : 16);
  prm.ksplit = pl.ksplit;
  prm.fmt = dtype == FML_F32 ? 2 : dtype == FML_BF16 ? 1 : 0;
  prm.p_mn = (pl.P.pack || pl.packed) ? 0 : (pl.P.mn ? 1 : 0);
  prm.q_mn = pl.Q.pack ? 0 : (pl.Q.mn ? 1 : 0);
  prm.swap = pl.swap ? 1 : 0;
  prm.out_dtype = dtype;
  prm.act = act;
  prm.stages = pl.stages;
  prm.esize = (int)es;
  prm.out = c;
  prm.ldo = ldc;
  prm.bias = bias;
  prm.bias_stride = bias_stride;
  prm.residual = residual;
  prm.ldr = ldr;
  prm.rows_out = (int)m;
  prm.cols_out = (int)n;
  prm.p_packed = p_packed;
  int red_stride = 0;
  const int smem = smem_bytes_for(pl.bn, pl.stages, pl.ksplit, &red_stride, pl.slabs, pl.pair, pl.fused);
  prm.red_stride = red_stride;
  prm.promote_kb = kPromoteKb;
  // Persistent grid (as many CTAs as are co-resident) without split-K; with
  // split-K one cluster per tile (the push reduction uses its receive
  // buffer once).
  const long long want = (long long)prm.num_tiles * prm.ksplit;
  int grid;
  if (pl.pair) {
    // one CTA per SM (the ring fills shared memory), whole pairs
    grid = (int)std::min<long long>((long long)prm.num_tiles * 2, (long long)(sms / 2) * 2);
  } else if (prm.ksplit > 1) {
    if (want > 0x7fffffffLL) return fail(FML_EUNSUPPORTED, "gemm: too many split-K tiles");
    grid = (int)want;
  } else {
    int res = resident_ctas(pl.bn, pl.promote, pl.ksplit, smem, sms);
    if (res <= 0) res = sms;
    grid = (int)std::min<long long>(want, res);
  }
  if (pl.fused) {
    // one tile per cluster: the LayerNorm prologue and the exchange run once per CTA
    if (grid < want) return fail(FML_EUNSUPPORTED, "linear_fused: output tiles exceed the co-resident CTAs");
    switch (pl.bn) {
      case 16: return launch_bn<16, false, false, true>(mp, mq, prm, grid, smem, st);
      case 32: return launch_bn<32, false, false, true>(mp, mq, prm, grid, smem, st);
    }
    return fail(FML_EUNSUPPORTED, "linear_fused: batch of more than 32 tokens");
  }
  if (pl.pair) return launch_bn<256, false, true>(mp, mq, prm, grid, smem, st);
  if (pl.promote) {
    switch (pl.bn) {
      case 16: return launch_bn<16, true>(mp, mq, prm, grid, smem, st);
      case 32: return launch_bn<32, true>(mp, mq, prm, grid, smem, st);
      case 64: return launch_bn<64, true>(mp, mq, prm, grid, smem, st);
    }
  } else {
    switch (pl.bn) {
      case 16: return launch_bn<16, false>(mp, mq, prm, grid, smem, st);
      case 32: return launch_bn<32, false>(mp, mq, prm, grid, smem, st);
      case 64: return launch_bn<64, false>(mp, mq, prm, grid, smem, st);
      case 128: return launch_bn<128, false>(mp, mq, prm, grid, smem, st);
      case 256: return launch_bn<256, false>(mp, mq, prm, grid, smem, st);
    }
  }
  return fail(FML_EUNSUPPORTED, "gemm: no kernel for tile width");
}

static int pack_operand(const Operand& o, int dtype, int mode, void* ws, cudaStream_t st) {
  dim3 blk(32, 8);
  const long long kp_w = o.kp;
  dim3 grd((unsigned)((kp_w + 31) / 32), (unsigned)((o.rows + 31) / 32));
  if (grd.y > 65535) return fail(FML_EUNSUPPORTED, "pack: too many rows");
  void* dst = static_cast<uint8_t*>(ws) + o.ws_off;
  if (dtype == FML_F32)
    launch_pdl(pack_kernel<float>, dim3(grd), dim3(blk), 0, st, 1, static_cast<const float*>(o.ptr), o.s_r, o.s_k,
                                            (int)o.rows, (int)o.k, (int)o.kp, mode,
                                            static_cast<float*>(dst));
  else if (dtype == FML_BF16)
    launch_pdl(pack_kernel<__nv_bfloat16>, dim3(grd), dim3(blk), 0, st, 1, 
        static_cast<const __nv_bfloat16*>(o.ptr), o.s_r, o.s_k, (int)o.rows, (int)o.k,
        (int)o.kp, 0, static_cast<__nv_bfloat16*>(dst));
  else
    launch_pdl(pack_kernel<__half>, dim3(grd), dim3(blk), 0, st, 1, static_cast<const __half*>(o.ptr), o.s_r, o.s_k,
                                             (int)o.rows, (int)o.k, (int)o.kp, 0,
                                             static_cast<__half*>(dst));
  count_launch();
  return check_cuda(cudaGetLastError(), "pack launch");
}

}  // namespace gemm
}  // namespace fml

using namespace fml;
using namespace fml::gemm;

static int validate_gemm(const void* a, const void* b, void* c, long long m, long long n,
                         long long k, int dtype) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "gemm: dtype must be f32, f16 or bf16");
  if (m <= 0 || n <= 0 || k <= 0) return fail(FML_EINVAL, "gemm: M, N, K must be positive");
  if (m > (1ll << 31) - 1 || n > (1ll << 31) - 1 || k > (1ll << 31) - 1)
    return fail(FML_EUNSUPPORTED, "gemm: dimension exceeds int32");
  if (!a || !b || !c) return fail(FML_EINVAL, "gemm: null operand pointer");
  return FML_OK;
}

// ---------------------------------------------------------------------------
// Plan cache of fml_gemm.  A plan (tile shape, split, residency, packing) and
// the two tensor maps depend only on the operands' addresses, layouts, the
// problem shape, dtype, tile hint, device and workspace address -- all in
// the key -- so a repeated call reuses them.  64 entries, replaced round
// robin; a tensor map is a function of its key, so an entry never goes stale.
// ---------------------------------------------------------------------------
struct PlanKey {
  const void* a;
  const void* b;
  const void* ws;
  long long v[7];  // lda_m, lda_k, ldb_k, ldb_n, m, n, k
  int dtype, dev;
  int cfg[5];      // -1 when no tile hint
  bool b_pre = false;  // b is a caller-packed 3xTF32 image
  bool operator==(const PlanKey& o) const {
    if (a != o.a || b != o.b || ws != o.ws || dtype != o.dtype || dev != o.dev || b_pre != o.b_pre) return false;
    for (int i = 0; i < 7; ++i)
      if (v[i] != o.v[i]) return false;
    for (int i = 0; i < 5; ++i)
      if (cfg[i] != o.cfg[i]) return false;
    return true;
  }
};

struct CachedPlan {
  alignas(64) CUtensorMap mp;
  alignas(64) CUtensorMap mq;
  PlanKey key;
  Plan pl;
  bool used = false;
};

static PlanKey plan_key(const void* a, long long lda_m, long long lda_k, const void* b, long long ldb_k,
                        long long ldb_n, long long m, long long n, long long k, int dtype, const fml_tile_cfg* cfg,
                        int dev, const void* ws) {
  PlanKey key;
  key.a = a;
  key.b = b;
  key.ws = ws;
  const long long v[7] = {lda_m, lda_k, ldb_k, ldb_n, m, n, k};
  for (int i = 0; i < 7; ++i) key.v[i] = v[i];
  key.dtype = dtype;
  key.dev = dev;
  const int c[5] = {cfg ? cfg->block_m : -1, cfg ? cfg->block_n : -1, cfg ? cfg->block_k : -1,
                    cfg ? cfg->num_warps : -1, cfg ? cfg->num_stages : -1};
  for (int i = 0; i < 5; ++i) key.cfg[i] = c[i];
  return key;
}

constexpr int kPlanCacheSize = 64;
static std::mutex g_plan_mu;
static CachedPlan g_plans[kPlanCacheSize];
static int g_plan_next = 0;

static bool plan_cache_get(const PlanKey& key, CachedPlan& out) {
  std::lock_guard<std::mutex> lock(g_plan_mu);
  for (int i = 0; i < kPlanCacheSize; ++i)
    if (g_plans[i].used && g_plans[i].key == key) {
      out = g_plans[i];
      return true;
    }
  return false;
}

static void plan_cache_put(const PlanKey& key, const Plan& pl, const CUtensorMap& mp, const CUtensorMap& mq) {
  std::lock_guard<std::mutex> lock(g_plan_mu);
  CachedPlan& e = g_plans[g_plan_next];
  g_plan_next = (g_plan_next + 1) % kPlanCacheSize;
  e.key = key;
  e.pl = pl;
  e.mp = mp;
  e.mq = mq;
  e.used = true;
}

extern "C" size_t fml_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int dtype,
                                          int64_t lda_m, int64_t lda_k, int64_t ldb_k,
                                          int64_t ldb_n, const void* a, const void* b,
                                          const fml_tile_cfg* cfg) {
  if (!valid_dtype(dtype) || m <= 0 || n <= 0 || k <= 0) return 0;
  Plan pl;
  const void* ap = a ? a : reinterpret_cast<const void*>(uintptr_t(256));
  const void* bp = b ? b : reinterpret_cast<const void*>(uintptr_t(256));
  if (make_plan(pl, ap, lda_m, lda_k, bp, ldb_k, ldb_n, m, n, k, dtype, cfg,
                num_sms(current_device())) != FML_OK)
    return 0;
  return pl.ws_bytes;
}

// Shared body of fml_gemm and fml_gemm_packed_b (b_pre: B's caller-packed
// 3xTF32 image, or null).
static int gemm_entry(const void* a, int64_t lda_m, int64_t lda_k, const void* b, int64_t ldb_k, int64_t ldb_n,
                      const void* b_pre, const void* bias, int64_t bias_stride, const void* residual, int64_t ldr,
                      void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype, int act,
                      const fml_tile_cfg* cfg, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_gemm(a, b, c, m, n, k, dtype);
  if (rc) return rc;
  if (act < 0 || act > 2) return fail(FML_EINVAL, "gemm: act must be 0 (none), 1 (erf) or 2 (tanh)");
  if (ldc < n) return fail(FML_EINVAL, "gemm: ldc < N");
  if (residual && ldr < n) return fail(FML_EINVAL, "gemm: ldr < N");
  if (cfg) {
    if (cfg->block_n < 0 || cfg->block_n > 256 || cfg->num_stages < 0 || cfg->num_stages > 16)
      return fail(FML_EINVAL, "gemm: tile config out of range");
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int dev = current_device();
  const int sms = num_sms(dev);
  PlanKey key = plan_key(a, lda_m, lda_k, b, ldb_k, ldb_n, m, n, k, dtype, cfg, dev, workspace);
  key.b_pre = b_pre != nullptr;
  CachedPlan hit;
  if (plan_cache_get(key, hit)) {
    // A repeated call (same operands, layout and workspace): the plan and
    // both tensor maps are the ones built before; only the packing kernels
    // (operand contents may have changed) and the launch run again.
    if (hit.pl.P.pack && (rc = pack_operand(hit.pl.P, dtype, split_mode(hit.pl.swap, dtype), workspace, st)))
      return rc;
    if (hit.pl.Q.pack && (rc = pack_operand(hit.pl.Q, dtype, split_mode(!hit.pl.swap, dtype), workspace, st)))
      return rc;
    return launch_plan(hit.pl, hit.mp, hit.mq, dtype, act, bias, bias_stride, residual, ldr, c, ldc, m, n, nullptr,
                       sms, st);
  }
  Plan pl;
  rc = make_plan(pl, a, lda_m, lda_k, b, ldb_k, ldb_n, m, n, k, dtype, cfg, sms, b_pre);
  if (rc) return rc;
  if (pl.ws_bytes > 0 && (workspace == nullptr || workspace_bytes < pl.ws_bytes))
    return fail(FML_EWORKSPACE, "gemm: workspace of " + std::to_string(pl.ws_bytes) +
                                    " bytes required");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) % 256) != 0)
    return fail(FML_EINVAL, "gemm: workspace must be 256-byte aligned");
  const bool tf32 = dtype == FML_F32;
  // Pack operands that TMA cannot read directly.
  if (pl.P.pack) {
    rc = pack_operand(pl.P, dtype, split_mode(pl.swap, dtype), workspace, st);
    if (rc) return rc;
  }
  if (pl.Q.pack) {
    rc = pack_operand(pl.Q, dtype, split_mode(!pl.swap, dtype), workspace, st);
    if (rc) return rc;
  }
  CUtensorMap mp, mq;
  for (int w = 0; w < 2; ++w) {
    Operand& o = w == 0 ? pl.P : pl.Q;
    CUtensorMap* map = w == 0 ? &mp : &mq;
    const int box_rows = w == 0 ? kBM : (pl.pair ? pl.bn / 2 : pl.bn);
    if (o.pre) {
      rc = encode(map, o.pre, dtype, tf32, false, o.rows, pl.keff, 3 * o.kp, box_rows);
    } else if (o.pack) {
      const void* ptr = static_cast<uint8_t*>(workspace) + o.ws_off;
      rc = encode(map, ptr, dtype, tf32, false, o.rows, pl.keff, tf32 ? 3 * o.kp : o.kp,
                  box_rows);
    } else if (!o.mn) {
      rc = encode(map, o.ptr, dtype, tf32, false, o.rows, pl.keff, o.s_r, box_rows);
    } else {
      rc = encode(map, o.ptr, dtype, tf32, true, o.rows, pl.keff, o.s_k, box_rows);
    }
    if (rc) return rc;
  }
  plan_cache_put(key, pl, mp, mq);
  return launch_plan(pl, mp, mq, dtype, act, bias, bias_stride, residual, ldr, c, ldc, m, n, nullptr, sms, st);
}

extern "C" int fml_gemm(const void* a, int64_t lda_m, int64_t lda_k, const void* b,
                        int64_t ldb_k, int64_t ldb_n, const void* bias, int64_t bias_stride,
                        const void* residual, int64_t ldr, void* c, int64_t ldc, int64_t m,
                        int64_t n, int64_t k, int dtype, int act, const fml_tile_cfg* cfg,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_entry(a, lda_m, lda_k, b, ldb_k, ldb_n, nullptr, bias, bias_stride, residual, ldr, c, ldc, m, n, k,
                    dtype, act, cfg, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// fp32 constant B operands split once (3xTF32 image [N, 3*Kp], hi|lo|hi).
// ---------------------------------------------------------------------------
static long long f32_kp(long long k) { return round_up(k, 4); }

extern "C" size_t fml_gemm_packed_b_bytes(int64_t n, int64_t k, int dtype) {
  if (dtype != FML_F32 || n <= 0 || k <= 0) return 0;
  return (size_t)round_up(n * 3 * f32_kp(k) * 4, 256);
}

extern "C" int fml_gemm_pack_b(const void* b, int64_t ldb_k, int64_t ldb_n, int64_t k, int64_t n, int dtype,
                               void* dst, size_t dst_bytes, void* stream) {
  if (dtype != FML_F32) return fail(FML_EUNSUPPORTED, "gemm_pack_b: fp32 only (16-bit B needs no split)");
  if (!b || !dst) return fail(FML_EINVAL, "gemm_pack_b: null pointer");
  if (n <= 0 || k <= 0) return fail(FML_EINVAL, "gemm_pack_b: N and K must be positive");
  if (n > (1ll << 31) - 1 || k > (1ll << 31) - 1) return fail(FML_EUNSUPPORTED, "gemm_pack_b: dimension exceeds int32");
  if (reinterpret_cast<uintptr_t>(dst) % 256 != 0) return fail(FML_EINVAL, "gemm_pack_b: dst must be 256-byte aligned");
  if (dst_bytes < fml_gemm_packed_b_bytes(n, k, dtype))
    return fail(FML_EINVAL, "gemm_pack_b: dst smaller than fml_gemm_packed_b_bytes");
  Operand o{b, ldb_n, ldb_k, n, k, false, true, 0, f32_kp(k)};
  return pack_operand(o, dtype, split_mode(true, dtype), dst, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t fml_gemm_packed_b_workspace_size(int64_t m, int64_t n, int64_t k, int dtype, int64_t lda_m,
                                                   int64_t lda_k, const void* a, const fml_tile_cfg* cfg) {
  if (dtype != FML_F32 || m <= 0 || n <= 0 || k <= 0) return 0;
  Plan pl;
  const void* ap = a ? a : reinterpret_cast<const void*>(uintptr_t(256));
  const void* bp = reinterpret_cast<const void*>(uintptr_t(256));
  if (make_plan(pl, ap, lda_m, lda_k, bp, 0, 0, m, n, k, dtype, cfg, num_sms(current_device()), bp) != FML_OK)
    return 0;
  return pl.ws_bytes;
}

extern "C" int fml_gemm_packed_b(const void* a, int64_t lda_m, int64_t lda_k, const void* b_packed,
                                 const void* bias, int64_t bias_stride, const void* residual, int64_t ldr, void* c,
                                 int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype, int act,
                                 const fml_tile_cfg* cfg, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != FML_F32) return fail(FML_EUNSUPPORTED, "gemm_packed_b: fp32 only");
  if (b_packed && reinterpret_cast<uintptr_t>(b_packed) % 256 != 0)
    return fail(FML_EINVAL, "gemm_packed_b: packed B must be 256-byte aligned");
  return gemm_entry(a, lda_m, lda_k, b_packed, 0, 0, b_packed, bias, bias_stride, residual, ldr, c, ldc, m, n, k,
                    dtype, act, cfg, workspace, workspace_bytes, stream);
}

static long long packed_kb(long long k, int dtype) { return (k * (long long)dtype_size(dtype) + kSlab - 1) / kSlab; }

extern "C" size_t fml_packed_weight_bytes(int64_t n, int64_t k, int dtype) {
  if (dtype != FML_BF16 && dtype != FML_F16) return 0;
  if (n <= 0 || k <= 0) return 0;
  return (size_t)((n + kBM - 1) / kBM) * (size_t)packed_kb(k, dtype) * (size_t)(kBM * kSlab);
}

extern "C" int fml_pack_weight(const void* w, int64_t ldw, int64_t n, int64_t k, int dtype, void* packed,
                               void* stream) {
  if (dtype != FML_BF16 && dtype != FML_F16)
    return fail(FML_EUNSUPPORTED, "pack_weight: 16-bit weights only (fp32 runs the 3xTF32 path)");
  if (!w || !packed) return fail(FML_EINVAL, "pack_weight: null pointer");
  if (n <= 0 || k <= 0 || ldw < k) return fail(FML_EINVAL, "pack_weight: bad shape");
  if (reinterpret_cast<uintptr_t>(packed) % 1024 != 0)
    return fail(FML_EINVAL, "pack_weight: packed buffer must be 1024-byte aligned");
  const long long nkb = packed_kb(k, dtype);
  const long long total = ((n + kBM - 1) / kBM) * nkb * (kBM * 8);
  const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 64);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FML_BF16)
    launch_pdl(pack_weight_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, 1, static_cast<const __nv_bfloat16*>(w), ldw, (int)n,
                                                            (int)k, (int)nkb, total, static_cast<uint8_t*>(packed));
  else
    launch_pdl(pack_weight_kernel<__half>, dim3(grid), dim3(256), 0, st, 1, static_cast<const __half*>(w), ldw, (int)n, (int)k, (int)nkb,
                                                     total, static_cast<uint8_t*>(packed));
  count_launch();
  return check_cuda(cudaGetLastError(), "pack_weight launch");
}

// MMA-space plan of a packed-weight product: P = packed W (N rows), Q = x
// (M rows), always the swapped form.
static int packed_plan(Plan& pl, const void* x, long long ldx, const void* packed, long long n, long long k,
                       long long m, int dtype, const fml_tile_cfg* cfg, int sms, bool fused) {
  pl.packed = true;
  pl.fused = fused;
  pl.swap = true;
  pl.promote = false;
  pl.P = Operand{packed, 0, 1, n, k, false, false, 0, 0};
  pl.Q = Operand{x, ldx, 1, m, k, false, false, 0, 0};
  pl.bn = pick_bn(pl, n, m, cfg, sms);
  classify(pl.Q, dtype, pl.bn, false);
  if (pl.Q.pack) return fail(FML_EUNSUPPORTED, "linear_packed: x must be row-major with 16-byte aligned rows");
  pl.keff = k;
  pl.ws_bytes = 0;
  pl.slabs = slabs_for(cfg, dtype, false, pl.bn, true);
  const long long tiles = ((n + kBM - 1) / kBM) * ((m + pl.bn - 1) / pl.bn);
  choose_split(pl, tiles, packed_kb(k, dtype), cfg, sms);
  return FML_OK;
}

extern "C" int fml_linear_packed(const void* x, int64_t ldx, const void* packed, int64_t n, int64_t k,
                                 const void* bias, int64_t bias_stride, const void* residual, int64_t ldr,
                                 void* out, int64_t ldo, int64_t m, int dtype, int act,
                                 const fml_tile_cfg* cfg, void* stream) {
  if (dtype != FML_BF16 && dtype != FML_F16) return fail(FML_EUNSUPPORTED, "linear_packed: 16-bit only");
  int rc = validate_gemm(x, packed, out, m, n, k, dtype);
  if (rc) return rc;
  if (act < 0 || act > 2) return fail(FML_EINVAL, "linear_packed: bad act");
  if (ldo < n || (residual && ldr < n) || (m > 1 && ldx < k))
    return fail(FML_EINVAL, "linear_packed: bad leading dimension");
  if (reinterpret_cast<uintptr_t>(packed) % 1024 != 0)
    return fail(FML_EINVAL, "linear_packed: packed weight must be 1024-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int sms = num_sms(current_device());
  Plan pl;
  rc = packed_plan(pl, x, ldx, packed, n, k, m, dtype, cfg, sms, false);
  if (rc) return rc;
  CUtensorMap mq;
  rc = encode(&mq, x, dtype, false, false, m, k, pl.Q.s_r, pl.bn);
  if (rc) return rc;
  return launch_plan(pl, mq, mq, dtype, act, bias, bias_stride, residual, ldr, out, ldo, m, n,
                     static_cast<const uint8_t*>(packed), sms, st);
}

// Whether the FUSED kernel covers the shape: 16-bit, m <= 32 (BN 16 or 32),
// one slab per stage, and one output tile per cluster with every CTA
// resident at once.
static bool fused_plan_ok(const Plan& pl, long long n, long long m, int sms) {
  if (pl.bn > 32 || pl.slabs != 1) return false;  // the LayerNorm prologue fills one slab per stage
  const long long tiles = ((n + kBM - 1) / kBM) * ((m + pl.bn - 1) / pl.bn);
  // Every CTA resident at once: the all-reduce epilogue waits on the other
  // ranks' CTAs of the same tile, which must not queue behind waiting CTAs.
  const int smem = smem_bytes_for(pl.bn, pl.stages, pl.ksplit, nullptr, pl.slabs, false, true);
  const int res = resident_ctas(pl.bn, false, pl.ksplit, smem, sms);
  return res > 0 && tiles * pl.ksplit <= res;
}

extern "C" int neb_linear_fused_ok(int64_t n, int64_t k, int64_t m, int dtype) {
  if ((dtype != FML_BF16 && dtype != FML_F16) || n <= 0 || k <= 0 || m <= 0 || m > 32) return 0;
  const int sms = num_sms(current_device());
  Plan pl;
  const void* fake = reinterpret_cast<const void*>(uintptr_t(1024));
  if (packed_plan(pl, fake, k, fake, n, k, m, dtype, nullptr, sms, true) != FML_OK) return 0;
  return fused_plan_ok(pl, n, m, sms) ? 1 : 0;
}

extern "C" int neb_linear_fused(const void* x, int64_t ldx, const void* packed, int64_t n, int64_t k,
                                const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int dtype,
                                int act, const neb_fusion* fu, void* stream) {
  if (dtype != FML_BF16 && dtype != FML_F16) return fail(FML_EUNSUPPORTED, "linear_fused: 16-bit only");
  int rc = validate_gemm(x, packed, out, m, n, k, dtype);
  if (rc) return rc;
  if (!fu) return fail(FML_EINVAL, "linear_fused: null fusion descriptor");
  if (act < 0 || act > 2) return fail(FML_EINVAL, "linear_fused: bad act");
  if (m > 32) return fail(FML_EUNSUPPORTED, "linear_fused: more than 32 tokens");
  if (reinterpret_cast<uintptr_t>(packed) % 1024 != 0)
    return fail(FML_EINVAL, "linear_fused: packed weight must be 1024-byte aligned");
  if ((m > 1 && ldx < k) || (residual && ldr < n)) return fail(FML_EINVAL, "linear_fused: bad leading dimension");
  Params fz = {};
  const bool kv = fu->k_pool != nullptr;
  const bool ar = fu->ar_ctx != nullptr;
  if (fu->ln_gamma && fu->ln_wsum) return fail(FML_EINVAL, "linear_fused: give ln_gamma (prologue) or ln_wsum (fold), not both");
  if (fu->ln_wsum) {
    if (k % 64 != 0) return fail(FML_EUNSUPPORTED, "linear_fused: LayerNorm fold needs k a multiple of 64");
    if (reinterpret_cast<uintptr_t>(x) % 16 || (ldx * 2) % 16)
      return fail(FML_EUNSUPPORTED, "linear_fused: LayerNorm operands must be 16-byte aligned");
    fz.ln_mode = 2;
    fz.fold_s = fu->ln_wsum;
    fz.fold_c = fu->ln_wbias;
    fz.ln_x = x;
    fz.ln_ldx = ldx;
    fz.ln_eps = fu->ln_eps;
    fz.ln_k = (int)k;
  }
  if (fu->ln_gamma) {
    if (!fu->ln_beta) return fail(FML_EINVAL, "linear_fused: LayerNorm needs gamma and beta");
    if (k % 64 != 0) return fail(FML_EUNSUPPORTED, "linear_fused: LayerNorm prologue needs k a multiple of 64");
    if (reinterpret_cast<uintptr_t>(x) % 16 || (ldx * 2) % 16 || reinterpret_cast<uintptr_t>(fu->ln_gamma) % 16 ||
        reinterpret_cast<uintptr_t>(fu->ln_beta) % 16)
      return fail(FML_EUNSUPPORTED, "linear_fused: LayerNorm operands must be 16-byte aligned");
    fz.ln_mode = 1;
    fz.ln_x = x;
    fz.ln_ldx = ldx;
    fz.ln_g = fu->ln_gamma;
    fz.ln_b = fu->ln_beta;
    fz.ln_eps = fu->ln_eps;
    fz.ln_k = (int)k;
  }
  if (kv) {
    if (!fu->v_pool || !fu->slot_of || !fu->start_pos) return fail(FML_EINVAL, "linear_fused: KV epilogue pointers");
    if (fu->q_cols < 0 || fu->kv_heads <= 0 || fu->head_dim <= 0 || fu->max_seq <= 0 || fu->tq <= 0 ||
        m % fu->tq != 0 || (long long)fu->q_cols + 2LL * fu->kv_heads * fu->head_dim != n)
      return fail(FML_EINVAL, "linear_fused: KV epilogue shape (n must be q_cols + 2*kv_heads*head_dim)");
    if (ldo < fu->q_cols) return fail(FML_EINVAL, "linear_fused: ldo < q_cols");
    if (fu->q_cols % 8 != 0 || fu->head_dim % 8 != 0 || reinterpret_cast<uintptr_t>(fu->k_pool) % 16 ||
        reinterpret_cast<uintptr_t>(fu->v_pool) % 16)
      return fail(FML_EUNSUPPORTED, "linear_fused: KV epilogue needs q_cols and head_dim multiples of 8, aligned pools");
    if (ar) return fail(FML_EUNSUPPORTED, "linear_fused: the KV and all-reduce epilogues do not combine");
    fz.kv_k = fu->k_pool;
    fz.kv_v = fu->v_pool;
    fz.kv_slot = fu->slot_of;
    fz.kv_start = fu->start_pos;
    fz.kv_q_cols = fu->q_cols;
    fz.kv_cols = fu->kv_heads * fu->head_dim;
    fz.kv_heads = fu->kv_heads;
    fz.kv_hd = fu->head_dim;
    fz.kv_max_seq = fu->max_seq;
    fz.kv_tq = fu->tq;
  } else if (ldo < n) {
    return fail(FML_EINVAL, "linear_fused: ldo < n");
  }
  if (ar) {
    const peer::Ctx* c = static_cast<const peer::Ctx*>(fu->ar_ctx);
    if (act != 0) return fail(FML_EUNSUPPORTED, "linear_fused: the all-reduce epilogue takes no activation");
    if (n % peer::kSubFeatures != 0 || n / peer::kSubFeatures > c->v.lay.nsub ||
        n * peer::kSubTokens * 2 > c->v.lay.slot_bytes)
      return fail(FML_EUNSUPPORTED, "linear_fused: n must be a multiple of 16 with n*64 <= the context's max_bytes");
    for (int q = 0; q < c->v.lay.world; ++q)
      if (!c->v.base[q]) return fail(FML_EINVAL, "linear_fused: all-reduce peers not opened");
    fz.ar_on = 1;
    fz.ar = c->v;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int sms = num_sms(current_device());
  Plan pl;
  rc = packed_plan(pl, x, ldx, packed, n, k, m, dtype, nullptr, sms, true);
  if (rc) return rc;
  if (!fused_plan_ok(pl, n, m, sms))
    return fail(FML_EUNSUPPORTED, "linear_fused: shape not covered (see neb_linear_fused_ok)");
  CUtensorMap mq;
  rc = encode(&mq, x, dtype, false, false, m, k, pl.Q.s_r, pl.bn);
  if (rc) return rc;
  return launch_plan(pl, mq, mq, dtype, act, nullptr, 0, residual, ldr, out, ldo, m, n,
                     static_cast<const uint8_t*>(packed), sms, st, &fz);
}

// ---------------------------------------------------------------------------
// fml_gemm_noalloc: the GEMM for callers that cannot allocate device memory.
// Its packing scratch is this file-scope device array instead of a caller
// workspace.  In host code the symbol is only a stand-in: the device address
// is looked up once per device with cudaGetSymbolAddress (that device
// current) and passed to the kernels like any workspace pointer.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[FML_GEMM_NOALLOC_SCRATCH_BYTES];

static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(FML_EUNSUPPORTED, "gemm_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "gemm_noalloc: cudaGetSymbolAddress");
    if (rc != FML_OK) return rc;
    addr[dev] = p;
  }
  *out = addr[dev];
  return FML_OK;
}

extern "C" int fml_gemm_noalloc(const void* a, int64_t lda_m, int64_t lda_k, const void* b, int64_t ldb_k,
                                int64_t ldb_n, const void* bias, int64_t bias_stride, const void* residual,
                                int64_t ldr, void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, int dtype,
                                int act, const fml_tile_cfg* cfg, void* stream) {
  int rc = validate_gemm(a, b, c, m, n, k, dtype);
  if (rc) return rc;
  const size_t need = fml_gemm_workspace_size(m, n, k, dtype, lda_m, lda_k, ldb_k, ldb_n, a, b, cfg);
  if (need > (size_t)FML_GEMM_NOALLOC_SCRATCH_BYTES)
    return fail(FML_EWORKSPACE, "gemm_noalloc: this problem needs " + std::to_string(need) +
                                    " bytes of packing scratch, more than the " +
                                    std::to_string((size_t)FML_GEMM_NOALLOC_SCRATCH_BYTES) +
                                    "-byte static scratch; use fml_gemm with a caller workspace");
  void* scratch = nullptr;
  if (need > 0) {
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
  }
  return fml_gemm(a, lda_m, lda_k, b, ldb_k, ldb_n, bias, bias_stride, residual, ldr, c, ldc, m, n, k, dtype, act,
                  cfg, scratch, need > 0 ? (size_t)FML_GEMM_NOALLOC_SCRATCH_BYTES : 0, stream);
}
