// Scaled-dot-product attention on the tcgen05 tensor cores (16-bit q, k, v):
//
//   out[b,h,i,:] = softmax_j(scale * q[b,h,i,:] . k[b,h,j,:]  (j <= i if causal)) v[b,h,j,:]
//
// the computation of torch's F.scaled_dot_product_attention that the
// reference evaluates for ForgeML's "sdpa" node (src/forgeml/ops.py:61-70)
// and that Nebula's prefill step writes out with a materialised score matrix
// (src/nebula/runtime.py:139-143).  Flash-attention schedule, one CTA per
// (batch, head, block of 128 queries), warp-specialised, 192 threads:
//
//   warp 4     TMA producer: the query tile once, then key / value tiles of
//              128 positions into a two-stage ring (4-D tensor maps over the
//              strided q/k/v views, so the wide QKV slot is read in place);
//   warp 5     TMEM owner and single-thread UMMA issuer:
//                S = Q K^T   (M = 128 queries, N = 128 keys, K = head dim)
//                O = P V     (M = 128 queries, N = head dim, K = 128 keys)
//              both bf16/fp16 in, fp32 accumulate in TMEM;
//   warps 0-3  softmax and epilogue, one query row per thread (its TMEM
//              lane): running max and sum in fp32, P = exp(S - max) written
//              as 16-bit values into shared memory in the swizzled UMMA
//              operand layout.  P V accumulates over the key blocks in TMEM;
//              when a row's maximum moves its TMEM output is scaled in place
//              (a warp whose rows all kept their maximum skips that), and the
//              normalised row is read out and stored once at the end.
//              Key blocks every row of a warp sees whole take an unmasked
//              path (MUFU exp2, packed 16-bit conversion, four independent
//              partial sums).
//
// Every wait is bounded (DEV_ERR_ATTN_TIMEOUT); a CTA that gives up lets its
// copies land and frees its TMEM before it exits.
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"

namespace fml {
namespace sdpa_tc {

constexpr int kThreads = 192;
constexpr int kBQ = 128;           // queries per CTA (UMMA M, TMEM lanes)
constexpr int kBK = 128;           // keys per block (UMMA N of S, K of P V)
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
// Dynamic shared memory beyond the layout: alignment of its base to 1024
// bytes.  Dynamic shared memory starts at least 512-byte aligned here (the
// kernel checks); 512 bytes keep two head-dim-64 CTAs within one SM.
constexpr uint32_t kAlignSlack = 512;
constexpr uint32_t kTmemCols = 256;  // S: 128 columns, the running O: head-dim columns

struct Args {
  int Sq, Sk, H;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  long long os[4];   // output strides (elements) of [B, H, Sq, D]
  // Nebula prefill over the KV pool (null for plain SDPA): request b's keys
  // are rows 0 .. start_pos[b] + Sq - 1 of pool slot slot_of[b], and its
  // query i sits at absolute position start_pos[b] + i (causal over
  // absolute positions, src/nebula/runtime.py:139-143).
  const int32_t* slot_of;
  const int32_t* start_pos;
  int max_seq;
};

// Coordinates of a tile in a 4-D tensor map whose outer dimensions are S, H
// and B in some order (dimension 0 is the head dim).
struct MapOrder {
  int s_dim, h_dim, b_dim;  // 1..3
};

template <int D>
struct Smem {
  static constexpr int kSlabs = D / 64;                 // 128-byte slabs along the head dim
  static constexpr uint32_t kTile = kBQ * D * 2;        // one q / k / v tile
  static constexpr uint32_t kP = kBQ * kBK * 2;         // the probabilities tile
  static constexpr uint32_t q = 0;
  static constexpr uint32_t kv = kTile;                 // stage s: K at kv + s * 2 * kTile, V after it
  static constexpr uint32_t p = kTile + 4 * kTile;
  static constexpr uint32_t bars = p + kP;              // 8-byte mbarriers, then the TMEM address
  static constexpr uint32_t total = bars + 128;
};

enum Bar : int { kQFull = 0, kKvFull0 = 1, kKvEmpty0 = 3, kSFull = 5, kPFull = 6, kOFull = 7, kNumBars = 8 };

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint32_t bar, uint32_t dst, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Tile coordinates (head-dim offset x, position s, head h, batch b) in the
// map's dimension order.
__device__ __forceinline__ void load_tile(const CUtensorMap* map, const MapOrder& o, uint32_t bar, uint32_t dst,
                                          int x, int s, int h, int b) {
  auto at = [&](int dim) { return o.s_dim == dim ? s : o.h_dim == dim ? h : b; };
  tma_load_4d(map, bar, dst, x, at(1), at(2), at(3));
}

// 2^x by the MUFU instruction (PTX ex2.approx.ftz.f32: a few ulp; the
// probabilities are rounded to 16 bits right after).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two probabilities as one packed 16-bit pair (first in the low half), and
// back to floats: the values the tensor core multiplies.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    return __half22float2(*reinterpret_cast<__half2*>(&w));
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, D <= 64 ? 2 : 1)
    sdpa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const MapOrder ord_q, const MapOrder ord_k,
                   const MapOrder ord_v, const Args a) {
  using L = Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The swizzled tiles want a 1024-byte aligned base; the launch adds
  // kAlignSlack bytes for that, enough for any 512-byte aligned start.
  if ((smem_u32(smem_raw) & 511u) != 0) {  // uniform: nothing touched yet
    if (threadIdx.x == 0) raise_device_error(DEV_ERR_ATTN_RANGE);
    return;
  }
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qblk = blockIdx.x, h = blockIdx.y % a.H, b = blockIdx.y / a.H;
  const int q0 = qblk * kBQ;
  auto bar = [&](int i) { return base + L::bars + 8u * (uint32_t)i; };
  const uint32_t tmem_holder = base + L::bars + 8u * kNumBars;
  // Keys of this request and the absolute position of its first query.
  // Pool slots and start positions are step inputs (no kernel of this
  // library writes them), so they are read before the dependency wait.
  int kv_b = b, q_off = 0, sk = a.Sk;
  if (a.slot_of != nullptr) {
    kv_b = a.slot_of[b];
    q_off = a.start_pos[b];
    sk = q_off + a.Sq;
    if (kv_b < 0 || q_off < 0 || sk > a.max_seq) {  // uniform over the CTA: no TMEM or barrier touched yet
      if (threadIdx.x == 0 && qblk == 0 && h == 0) raise_device_error(DEV_ERR_ATTN_RANGE);
      return;
    }
  }
  // keys this block of queries attends to
  const int kend = a.causal ? min(sk, q0 + kBQ + q_off) : sk;
  const int nkb = (kend + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kKvFull0 + s), 1);
      mbar_init(bar(kKvEmpty0 + s), 1);
    }
    mbar_init(bar(kSFull), 1);
    mbar_init(bar(kPFull), 4);  // one arrive per softmax warp
    mbar_init(bar(kOFull), 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  uint32_t tmem;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem) : "r"(tmem_holder) : "memory");

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
    }
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      int issued = 0;  // K/V stages whose loads were issued
      mbar_arrive_expect_tx(bar(kQFull), L::kTile);
      for (int sl = 0; sl < L::kSlabs; ++sl)
        load_tile(&tmQ, ord_q, bar(kQFull), base + L::q + sl * kBQ * 128, sl * 64, q0, h, b);
      bool ok = true;
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(bar(kKvEmpty0 + st), ((j >> 1) - 1) & 1, DEV_ERR_ATTN_TIMEOUT)) {
          ok = false;
          break;
        }
        const uint32_t kdst = base + L::kv + st * 2 * L::kTile, vdst = kdst + L::kTile;
        mbar_arrive_expect_tx(bar(kKvFull0 + st), 2 * L::kTile);
        for (int sl = 0; sl < L::kSlabs; ++sl) {
          load_tile(&tmK, ord_k, bar(kKvFull0 + st), kdst + sl * kBK * 128, sl * 64, j * kBK, h, kv_b);
          load_tile(&tmV, ord_v, bar(kKvFull0 + st), vdst + sl * kBK * 128, sl * 64, j * kBK, h, kv_b);
        }
        ++issued;
      }
      if (!ok) {
        // let the loads already issued land before the CTA may exit
        mbar_wait(bar(kQFull), 0, DEV_ERR_ATTN_TIMEOUT);
        for (int j = max(0, issued - 2); j < issued; ++j)
          mbar_wait(bar(kKvFull0 + (j & 1)), (j >> 1) & 1, DEV_ERR_ATTN_TIMEOUT);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ UMMA issuer
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      const int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t id_s = umma_idesc(fmt, 0, 0, kBK);  // Q (K-major) x K (K-major)
      const uint32_t id_o = umma_idesc(fmt, 0, 1, D);    // P (K-major) x V (MN-major along the head dim)
      const uint64_t dq = umma_desc_sw128(base + L::q, 16u, 1024u);
      const uint64_t dp = umma_desc_sw128(base + L::p, 16u, 1024u);
      bool okk = mbar_wait(bar(kQFull), 0, DEV_ERR_ATTN_TIMEOUT);
      int done = 0;     // blocks whose P V was issued
      int s_issued = 0; // blocks whose Q K^T was issued
      for (int j = 0; j < nkb && okk; ++j) {
        const int st = j & 1;
        if (!mbar_wait(bar(kKvFull0 + st), (j >> 1) & 1, DEV_ERR_ATTN_TIMEOUT)) { okk = false; break; }
        tc_fence_after();
        const uint32_t kaddr = base + L::kv + st * 2 * L::kTile, vaddr = kaddr + L::kTile;
        const uint64_t dk = umma_desc_sw128(kaddr, 16u, 1024u);
        const uint64_t dv = umma_desc_sw128(vaddr, (uint32_t)(kBK * 128), 1024u);
        // S = Q K^T over the head dim: per slab 4 steps of 16 elements (32 bytes)
#pragma unroll
        for (int sl = 0; sl < L::kSlabs; ++sl)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t off = (uint32_t)(sl * kBQ * 128 + k * 32) >> 4;
            umma_f16(tmem, dq + off, dk + off, id_s, (sl | k) != 0);
          }
        umma_commit(bar(kSFull));
        s_issued = j + 1;
        // O += P V once the softmax warps wrote P (and rescaled O where needed)
        if (!mbar_wait(bar(kPFull), j & 1, DEV_ERR_ATTN_TIMEOUT)) { okk = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // P: 16 keys = 32 bytes within a 64-key slab; V: 16 key rows of 128 bytes
          const uint32_t poff = (uint32_t)((k / 4) * kBQ * 128 + (k % 4) * 32) >> 4;
          const uint32_t voff = (uint32_t)(k * 16 * 128) >> 4;
          umma_f16(tmem + kBK, dp + poff, dv + voff, id_o, (j | k) != 0);  // O accumulates over the blocks
        }
        umma_commit(bar(kOFull));
        umma_commit(bar(kKvEmpty0 + st));
        done = j + 1;
      }
      // every UMMA issued above completes before TMEM is released: the last
      // Q K^T commit and the last P V commit
      if (s_issued > 0) mbar_wait(bar(kSFull), (s_issued - 1) & 1, DEV_ERR_ATTN_TIMEOUT);
      if (done > 0) mbar_wait(bar(kOFull), (done - 1) & 1, DEV_ERR_ATTN_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    pdl_wait();
    pdl_trigger();
    const int r = threadIdx.x;  // query row in the block = TMEM lane
    const int qi = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool live = true;
    for (int j = 0; j < nkb; ++j) {
      live = live && mbar_wait(bar(kSFull), j & 1, DEV_ERR_ATTN_TIMEOUT);
      tc_fence_after();
      const int key0 = j * kBK;
      // keys of this block this row may see
      int lim = min(kBK, sk - key0);
      if (a.causal) lim = min(lim, qi + q_off - key0 + 1);
      // every row of the warp sees the whole block: no per-key masking
      const bool full = __all_sync(0xffffffffu, lim >= kBK);
      // pass 1: row maximum of the scaled scores
      float mx = -INFINITY;
      if (full) {
#pragma unroll
        for (int c = 0; c < kBK / 32; ++c) {
          float v[32];
          tmem_ld32(trow + c * 32, v);
          float m2[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
          for (int e = 4; e < 32; ++e) m2[e & 3] = fmaxf(m2[e & 3], v[e]);
          mx = fmaxf(mx, fmaxf(fmaxf(m2[0], m2[1]), fmaxf(m2[2], m2[3])));
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBK / 32; ++c) {
          float v[32];
          tmem_ld32(trow + c * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e < lim) mx = fmaxf(mx, v[e]);
        }
      }
      const float m_new = fmaxf(m, mx * a.scale_log2);
      // The running output lives in TMEM (P V accumulates into it).  Once
      // the previous block's P V has landed, rows whose maximum moved scale
      // their output in place; a warp whose rows all kept theirs skips it.
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
      if (j > 0) {
        live = live && mbar_wait(bar(kOFull), (j - 1) & 1, DEV_ERR_ATTN_TIMEOUT);
        tc_fence_after();
        if (!__all_sync(0xffffffffu, alpha == 1.f)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float v[32];
            tmem_ld32(trow + kBK + c * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(trow + kBK + c * 32, v);
          }
        }
      }
      l *= alpha;
      m = m_new;
      // pass 2: probabilities, their sum, and P into the swizzled operand tile
      const uint32_t prow = base + L::p + (uint32_t)r * 128u;
      float lp[4] = {0.f, 0.f, 0.f, 0.f};  // partial sums (independent add chains)
#pragma unroll
      for (int c = 0; c < kBK / 32; ++c) {
        float v[32];
        tmem_ld32(trow + c * 32, v);
        uint32_t w[16];
        if (full) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            w[e / 2] = pack2<T>(ex2_approx(fmaf(v[e], a.scale_log2, -m)), ex2_approx(fmaf(v[e + 1], a.scale_log2, -m)));
            const float2 f = unpack2<T>(w[e / 2]);  // the sum of what the tensor core multiplies
            lp[(e / 2) & 3] += f.x + f.y;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = (c * 32 + e < lim && m != -INFINITY) ? exp2f(v[e] * a.scale_log2 - m) : 0.f;
            const float p1 = (c * 32 + e + 1 < lim && m != -INFINITY) ? exp2f(v[e + 1] * a.scale_log2 - m) : 0.f;
            T t0 = from_f32<T>(p0), t1 = from_f32<T>(p1);
            lp[0] += to_f32<T>(t0) + to_f32<T>(t1);
            w[e / 2] = (uint32_t)(*reinterpret_cast<uint16_t*>(&t0)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&t1)) << 16);
          }
        }
        // 32 keys = 4 chunks of 16 bytes, in slab (c / 2), chunks 4 * (c % 2) ..
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int chunk = 4 * (c % 2) + q4;
          const uint32_t addr = prow + (uint32_t)(c / 2) * (kBQ * 128) + (uint32_t)((chunk ^ (r & 7)) * 16);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * q4]),
                       "r"(w[4 * q4 + 1]), "r"(w[4 * q4 + 2]), "r"(w[4 * q4 + 3])
                       : "memory");
        }
      }
      l += (lp[0] + lp[1]) + (lp[2] + lp[3]);
      // Pool rows past this request's keys hold stale data (possibly not
      // finite) that P V would multiply by zero: clear them in the V tile.
      // (Outside the tensor map, as in plain SDPA, TMA fills zeros itself.)
      if (a.slot_of != nullptr && key0 + kBK > sk) {
        live = live && mbar_wait(bar(kKvFull0 + (j & 1)), (j >> 1) & 1, DEV_ERR_ATTN_TIMEOUT);
        if (key0 + r >= sk) {
          const uint32_t vrow = base + L::kv + (j & 1) * 2 * L::kTile + L::kTile + (uint32_t)r * 128u;
#pragma unroll
          for (int sl = 0; sl < L::kSlabs; ++sl)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vrow + sl * kBK * 128 + c * 16), "r"(0u)
                           : "memory");
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull));
    }
    // the output row: the accumulated P V from TMEM, normalised by the sum
    if (nkb > 0) {
      live = live && mbar_wait(bar(kOFull), (nkb - 1) & 1, DEV_ERR_ATTN_TIMEOUT);
      tc_fence_after();
    }
    const float inv = 1.0f / l;  // l == 0 (every key masked) gives NaN, as torch
    T* out = static_cast<T*>(a.out) + b * a.os[0] + h * a.os[1] + (long long)qi * a.os[2];
    const bool vec = a.os[3] == 1 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float v[32];
      if (nkb > 0) {
        tmem_ld32(trow + kBK + c * 32, v);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      if (!(live && qi < a.Sq)) continue;
      if (vec) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<uint4*>(out + c * 32)[q] =
              make_uint4(pack2<T>(v[8 * q] * inv, v[8 * q + 1] * inv), pack2<T>(v[8 * q + 2] * inv, v[8 * q + 3] * inv),
                         pack2<T>(v[8 * q + 4] * inv, v[8 * q + 5] * inv), pack2<T>(v[8 * q + 6] * inv, v[8 * q + 7] * inv));
      } else {
        for (int e = 0; e < 32; ++e) out[(long long)(c * 32 + e) * a.os[3]] = from_f32<T>(v[e] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// A 4-D map of one operand [B, H, S, D] (element strides st[0..3], st[3] == 1):
// dimension 0 is the head dim; the outer three are S, H and B ordered by
// increasing stride (the encoder wants each stride to cover the dimensions
// inside it).  Box: 64 head-dim elements (128 bytes, the swizzle span) x 128
// positions.  Returns false when the layout cannot be described.
static bool encode_operand(CUtensorMap* map, MapOrder* order, const void* ptr, const int64_t st[4], int64_t B,
                           int64_t H, int64_t S, int64_t D, bool bf16) {
  EncodeFn fn = encode_fn();
  if (!fn || st[3] != 1 || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  struct Dim {
    int which;  // 0 = S, 1 = H, 2 = B
    long long extent, stride;
  } dims[3] = {{0, S, st[2]}, {1, H, st[1]}, {2, B, st[0]}};
  // order by stride (extent-1 dimensions may sit anywhere: give them a stride that sorts last)
  for (int i = 0; i < 3; ++i)
    if (dims[i].extent == 1) dims[i].stride = (1LL << 40) / 2 + i;
  for (int i = 0; i < 3; ++i)
    for (int j = i + 1; j < 3; ++j)
      if (dims[j].stride < dims[i].stride) std::swap(dims[i], dims[j]);
  cuuint64_t gdim[4] = {(cuuint64_t)D, 0, 0, 0}, gstr[3];
  cuuint32_t box[4] = {64, 1, 1, 1}, estr[4] = {1, 1, 1, 1};
  long long covered = D * 2;  // bytes spanned by the dimensions inside
  for (int i = 0; i < 3; ++i) {
    const long long bytes = dims[i].stride * 2;
    if (dims[i].extent > 1 && (bytes % 16 != 0 || bytes < covered)) return false;
    const long long use = dims[i].extent > 1 ? bytes : covered;
    gdim[i + 1] = (cuuint64_t)dims[i].extent;
    gstr[i] = (cuuint64_t)((use + 15) / 16 * 16);
    covered = (long long)gstr[i] * dims[i].extent;
    if (dims[i].which == 0) box[i + 1] = (cuuint32_t)kBQ;
    (dims[i].which == 0 ? order->s_dim : dims[i].which == 1 ? order->h_dim : order->b_dim) = i + 1;
  }
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(ptr), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D>
static int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const MapOrder& oq,
                  const MapOrder& ok, const MapOrder& ov, const Args& a, int64_t B, int64_t H, cudaStream_t st) {
  const size_t smem = Smem<D>::total + kAlignSlack;
  cudaError_t e = cudaFuncSetAttribute(sdpa_tc_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "sdpa_tc attribute");
  const dim3 grid((unsigned)((a.Sq + kBQ - 1) / kBQ), (unsigned)(B * H));
  e = launch_pdl(sdpa_tc_kernel<T, D>, grid, dim3(kThreads), smem, st, 1, mq, mk, mv, oq, ok, ov, a);
  count_launch();
  return check_cuda(e, "sdpa_tc launch");
}

}  // namespace sdpa_tc

// Nebula prefill attention over the KV pool on the tensor cores: queries
// q [B, T, H, D] (strided), keys / values rows of pool [slots, H, max_seq, D]
// (contiguous), out [B, T, H*D] contiguous.  FML_EUNSUPPORTED when not
// covered (fp32, head dim other than 64 / 128, unaddressable strides).
int neb_prefill_tensor_core(const void* q, const int64_t qs[4], const void* k_pool, const void* v_pool,
                            const int32_t* slot_of, const int32_t* start_pos, void* out, int64_t B, int64_t T,
                            int64_t H, int64_t D, int64_t max_seq, int64_t slots, float scale, int dtype,
                            cudaStream_t st) {
  using namespace sdpa_tc;
  if ((dtype != FML_BF16 && dtype != FML_F16) || (D != 64 && D != 128)) return FML_EUNSUPPORTED;
  if (B * H > 65535 || max_seq > (1 << 30)) return FML_EUNSUPPORTED;
  const bool bf = dtype == FML_BF16;
  // q as [B, H, T, D]; the pools as [slots, H, max_seq, D]
  const int64_t q4[4] = {qs[0], qs[2], qs[1], qs[3]};
  const int64_t p4[4] = {H * max_seq * D, max_seq * D, D, 1};
  CUtensorMap mq, mk, mv;
  MapOrder oq{}, okk{}, ov{};
  if (!encode_operand(&mq, &oq, q, q4, B, H, T, D, bf) ||
      !encode_operand(&mk, &okk, k_pool, p4, slots, H, max_seq, D, bf) ||
      !encode_operand(&mv, &ov, v_pool, p4, slots, H, max_seq, D, bf))
    return FML_EUNSUPPORTED;
  Args a = {};
  a.Sq = (int)T;
  a.Sk = (int)max_seq;
  a.H = (int)H;
  a.causal = 1;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  const int64_t o4[4] = {T * H * D, D, H * D, 1};  // [B, T, H, D] seen as [B, H, T, D]
  for (int i = 0; i < 4; ++i) a.os[i] = o4[i];
  a.slot_of = slot_of;
  a.start_pos = start_pos;
  a.max_seq = (int)max_seq;
  if (bf)
    return D == 64 ? launch<__nv_bfloat16, 64>(mq, mk, mv, oq, okk, ov, a, B, H, st)
                   : launch<__nv_bfloat16, 128>(mq, mk, mv, oq, okk, ov, a, B, H, st);
  return D == 64 ? launch<__half, 64>(mq, mk, mv, oq, okk, ov, a, B, H, st)
                 : launch<__half, 128>(mq, mk, mv, oq, okk, ov, a, B, H, st);
}

// Runs the tensor-core kernel when it covers the call: 16-bit q/k/v/out,
// head dim 64 or 128, no explicit mask (causal allowed), unit head-dim
// strides, 16-byte aligned bases and row strides.  Returns FML_EUNSUPPORTED
// (nothing launched) otherwise.
int sdpa_tensor_core(const void* q, const int64_t qs[4], const void* k, const int64_t ks[4], const void* v,
                     const int64_t vs[4], int mask_kind, int is_causal, float scale, void* out,
                     const int64_t os[4], int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int dtype,
                     cudaStream_t st) {
  using namespace sdpa_tc;
  if ((dtype != FML_BF16 && dtype != FML_F16) || mask_kind != 0 || (D != 64 && D != 128)) return FML_EUNSUPPORTED;
  if (B * H > 65535 || Sq > (1 << 30) || Sk > (1 << 30)) return FML_EUNSUPPORTED;
  CUtensorMap mq, mk, mv;
  MapOrder oq{}, okk{}, ov{};
  const bool bf = dtype == FML_BF16;
  if (!encode_operand(&mq, &oq, q, qs, B, H, Sq, D, bf) || !encode_operand(&mk, &okk, k, ks, B, H, Sk, D, bf) ||
      !encode_operand(&mv, &ov, v, vs, B, H, Sk, D, bf))
    return FML_EUNSUPPORTED;
  Args a = {};
  a.Sq = (int)Sq;
  a.Sk = (int)Sk;
  a.H = (int)H;
  a.causal = is_causal ? 1 : 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  for (int i = 0; i < 4; ++i) a.os[i] = os[i];
  if (bf)
    return D == 64 ? launch<__nv_bfloat16, 64>(mq, mk, mv, oq, okk, ov, a, B, H, st)
                   : launch<__nv_bfloat16, 128>(mq, mk, mv, oq, okk, ov, a, B, H, st);
  return D == 64 ? launch<__half, 64>(mq, mk, mv, oq, okk, ov, a, B, H, st)
                 : launch<__half, 128>(mq, mk, mv, oq, okk, ov, a, B, H, st);
}

}  // namespace fml
