// Small Nebula decode-step kernels: KV-cache append, token + position
// embedding, greedy argmax and the residual add used after a tensor-parallel
// all-reduce.  All are HBM/latency-bound elementwise kernels with 16-byte
// vector accesses where the layout allows.
#include <cmath>
#include <string>

#include "common.cuh"

namespace fml {
namespace neb {

// pool[slot_of[b], h, start_pos[b]+t, :] = src[b, t, h, :] for K and V.
// One thread per 16-byte slice (vector path) or per element.
template <typename T, bool VEC>
__global__ void kv_append_kernel(const T* __restrict__ k, long long ks0, long long ks1, long long ks2,
                                 const T* __restrict__ v, long long vs0, long long vs1, long long vs2,
                                 T* __restrict__ kp, T* __restrict__ vp,
                                 const int32_t* __restrict__ slot_of,
                                 const int32_t* __restrict__ start_pos, int tq, int H, int D,
                                 int max_seq, long long total) {
  pdl_wait();
  pdl_trigger();
  constexpr int W = VEC ? (int)(16 / sizeof(T)) : 1;
  const int per_row = D / W;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % per_row);
    long long r = idx / per_row;
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % tq);
    const int b = (int)(r / tq);
    const int slot = slot_of[b];
    const int pos = start_pos[b] + t;
    if (slot < 0 || pos < 0 || pos >= max_seq) {
      raise_device_error(DEV_ERR_ATTN_RANGE);
      continue;
    }
    const long long dst = (((long long)slot * H + h) * max_seq + pos) * D + (long long)c * W;
    const long long sk = b * ks0 + (long long)t * ks1 + (long long)h * ks2 + (long long)c * W;
    const long long sv = b * vs0 + (long long)t * vs1 + (long long)h * vs2 + (long long)c * W;
    if (VEC) {
      *reinterpret_cast<uint4*>(kp + dst) = *reinterpret_cast<const uint4*>(k + sk);
      *reinterpret_cast<uint4*>(vp + dst) = *reinterpret_cast<const uint4*>(v + sv);
    } else {
      kp[dst] = k[sk];
      vp[dst] = v[sv];
    }
  }
}

// x[b,t,:] = round(tok_emb[tokens[b,t],:] + pos_emb[start_pos[b]+t,:])
template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ tokens, const int32_t* __restrict__ start_pos,
                             const T* __restrict__ te, const T* __restrict__ pe, T* __restrict__ x,
                             int tq, int hidden, long long vocab, int max_seq) {
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;  // b * tq + t
  const int b = (int)(row / tq), t = (int)(row % tq);
  const long long tok = tokens[row];
  const int pos = start_pos[b] + t;
  T* xr = x + row * hidden;
  if (tok < 0 || tok >= vocab || pos < 0 || pos >= max_seq) {
    if (threadIdx.x == 0) raise_device_error(DEV_ERR_TOKEN_RANGE);
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = from_f32<T>(0.f);
    return;
  }
  const T* tr = te + tok * hidden;
  const T* pr = pe + (long long)pos * hidden;
  constexpr int W = 16 / sizeof(T);
  if (hidden % W == 0) {
    for (int c = threadIdx.x * W; c < hidden; c += blockDim.x * W) {
      uint4 a = *reinterpret_cast<const uint4*>(tr + c);
      uint4 p = *reinterpret_cast<const uint4*>(pr + c);
      uint4 o;
      const T* ea = reinterpret_cast<const T*>(&a);
      const T* ep = reinterpret_cast<const T*>(&p);
      T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int i = 0; i < W; ++i) eo[i] = from_f32<T>(to_f32<T>(ea[i]) + to_f32<T>(ep[i]));
      *reinterpret_cast<uint4*>(xr + c) = o;
    }
  } else {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x)
      xr[c] = from_f32<T>(to_f32<T>(tr[c]) + to_f32<T>(pr[c]));
  }
}

// (value, index) ordering of torch.argmax: NaN is the maximum, ties go to the
// smallest index.
__device__ __forceinline__ bool better(float v, long long i, float bv, long long bi) {
  const bool vn = isnan(v), bn = isnan(bv);
  if (vn || bn) {
    if (vn && !bn) return true;
    if (!vn && bn) return false;
    return i < bi;
  }
  if (v > bv) return true;
  if (v < bv) return false;
  return i < bi;
}

// One CTA per row.  VEC: 16-byte loads, a thread's vectors all issued before
// any is compared (one memory latency per row instead of one per element).
template <typename T, bool VEC>
__global__ void __launch_bounds__(1024)
    argmax_kernel(const T* __restrict__ logits, long long rs, long long cols, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const T* row = logits + (long long)blockIdx.x * rs;
  float bv = -INFINITY;
  long long bi = cols;  // sentinel (worse than any real index once a value is seen)
  if (VEC) {
    constexpr int E = 16 / sizeof(T);
    constexpr int kBatch = 4;  // vectors in flight per thread
    const long long nvec = cols / E;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    for (long long v0 = threadIdx.x; v0 < nvec; v0 += (long long)kBatch * blockDim.x) {
      uint4 w[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const long long vi = v0 + (long long)u * blockDim.x;
        if (vi < nvec) w[u] = rv[vi];
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const long long vi = v0 + (long long)u * blockDim.x;
        if (vi >= nvec) continue;
        const T* e = reinterpret_cast<const T*>(&w[u]);
#pragma unroll
        for (int k = 0; k < E; ++k) {
          const float v = to_f32<T>(e[k]);
          const long long c = vi * E + k;
          if (bi == cols || better(v, c, bv, bi)) { bv = v; bi = c; }
        }
      }
    }
    for (long long c = nvec * E + threadIdx.x; c < cols; c += blockDim.x) {  // tail
      const float v = to_f32<T>(row[c]);
      if (bi == cols || better(v, c, bv, bi)) { bv = v; bi = c; }
    }
  } else {
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
      const float v = to_f32<T>(row[c]);
      if (bi == cols || better(v, c, bv, bi)) { bv = v; bi = c; }
    }
  }
  __shared__ float sv[32];
  __shared__ long long si[32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (oi != cols && (bi == cols || better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) / 32;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : cols;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi != cols && (bi == cols || better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) out[blockIdx.x] = bi;
  }
}

template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, long long n) {
  pdl_wait();
  pdl_trigger();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = from_f32<T>(to_f32<T>(a[i]) + to_f32<T>(b[i]));
}

static unsigned grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  if (g > 148LL * 32) g = 148LL * 32;
  return (unsigned)std::max<long long>(g, 1);
}

}  // namespace neb
}  // namespace fml

using namespace fml;

extern "C" int neb_kv_append(const void* k, const int64_t k_strides[4], const void* v,
                             const int64_t v_strides[4], void* k_pool, void* v_pool,
                             const int32_t* slot_of, const int32_t* start_pos, int64_t batch,
                             int64_t t, int64_t heads, int64_t head_dim, int64_t max_seq, int dtype,
                             void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "neb_kv_append: bad dtype");
  if (!k || !v || !k_pool || !v_pool || !slot_of || !start_pos || !k_strides || !v_strides)
    return fail(FML_EINVAL, "neb_kv_append: null pointer");
  if (batch <= 0 || t <= 0 || heads <= 0 || head_dim <= 0 || max_seq <= 0)
    return fail(FML_EINVAL, "neb_kv_append: sizes must be positive");
  if (k_strides[3] != 1 || v_strides[3] != 1)
    return fail(FML_EUNSUPPORTED, "neb_kv_append: innermost stride must be 1");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long es = (long long)dtype_size(dtype);
  const long long W = 16 / es;
  bool vec = (head_dim % W == 0);
  for (int i = 0; i < 3; ++i) vec = vec && (k_strides[i] % W == 0) && (v_strides[i] % W == 0);
  vec = vec && reinterpret_cast<uintptr_t>(k) % 16 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(k_pool) % 16 == 0 && reinterpret_cast<uintptr_t>(v_pool) % 16 == 0;
  const long long total = batch * t * heads * (vec ? head_dim / W : head_dim);
  const unsigned grid = neb::grid_for(total, 256);
#define KV_LAUNCH(TT, VV)                                                                         \
  launch_pdl(neb::kv_append_kernel<TT, VV>, dim3(grid), dim3(256), 0, st, 1,                                            \
      static_cast<const TT*>(k), k_strides[0], k_strides[1], k_strides[2],                        \
      static_cast<const TT*>(v), v_strides[0], v_strides[1], v_strides[2],                        \
      static_cast<TT*>(k_pool), static_cast<TT*>(v_pool), slot_of, start_pos, (int)t, (int)heads, \
      (int)head_dim, (int)max_seq, total)
  if (dtype == FML_F32) { if (vec) KV_LAUNCH(float, true); else KV_LAUNCH(float, false); }
  else if (dtype == FML_BF16) { if (vec) KV_LAUNCH(__nv_bfloat16, true); else KV_LAUNCH(__nv_bfloat16, false); }
  else { if (vec) KV_LAUNCH(__half, true); else KV_LAUNCH(__half, false); }
#undef KV_LAUNCH
  count_launch();
  return check_cuda(cudaGetLastError(), "neb_kv_append launch");
}

extern "C" int neb_embed(const int64_t* tokens, const int32_t* start_pos, const void* tok_emb,
                         const void* pos_emb, void* x, int64_t batch, int64_t t, int64_t hidden,
                         int64_t vocab, int64_t max_seq, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "neb_embed: bad dtype");
  if (!tokens || !start_pos || !tok_emb || !pos_emb || !x) return fail(FML_EINVAL, "neb_embed: null pointer");
  if (batch <= 0 || t <= 0 || hidden <= 0 || vocab <= 0 || max_seq <= 0)
    return fail(FML_EINVAL, "neb_embed: sizes must be positive");
  if (batch * t > (1ll << 31) - 1) return fail(FML_EUNSUPPORTED, "neb_embed: too many rows");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(batch * t);
  const bool al = reinterpret_cast<uintptr_t>(tok_emb) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(pos_emb) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
  if (!al) return fail(FML_EUNSUPPORTED, "neb_embed: tables and output must be 16-byte aligned");
  if (dtype == FML_F32)
    launch_pdl(neb::embed_kernel<float>, dim3(grid), dim3(256), 0, st, 1, tokens, start_pos, static_cast<const float*>(tok_emb),
        static_cast<const float*>(pos_emb), static_cast<float*>(x), (int)t, (int)hidden, vocab, (int)max_seq);
  else if (dtype == FML_BF16)
    launch_pdl(neb::embed_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, 1, tokens, start_pos,
        static_cast<const __nv_bfloat16*>(tok_emb), static_cast<const __nv_bfloat16*>(pos_emb),
        static_cast<__nv_bfloat16*>(x), (int)t, (int)hidden, vocab, (int)max_seq);
  else
    launch_pdl(neb::embed_kernel<__half>, dim3(grid), dim3(256), 0, st, 1, tokens, start_pos, static_cast<const __half*>(tok_emb),
        static_cast<const __half*>(pos_emb), static_cast<__half*>(x), (int)t, (int)hidden, vocab, (int)max_seq);
  count_launch();
  return check_cuda(cudaGetLastError(), "neb_embed launch");
}

extern "C" int neb_argmax(const void* logits, int64_t row_stride, int64_t rows, int64_t cols,
                          int64_t* out, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "neb_argmax: bad dtype");
  if (!logits || !out) return fail(FML_EINVAL, "neb_argmax: null pointer");
  if (rows <= 0 || cols <= 0 || rows > (1ll << 31) - 1) return fail(FML_EINVAL, "neb_argmax: bad sizes");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int threads = cols >= 1024 ? 1024 : 256;
  const long long es = (long long)dtype_size(dtype);
  const bool vec = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (row_stride * es) % 16 == 0;
#define ARGMAX_LAUNCH(TT)                                                                                       \
  (vec ? launch_pdl(neb::argmax_kernel<TT, true>, dim3((unsigned)rows), dim3(threads), 0, st, 1,              \
                    static_cast<const TT*>(logits), (long long)row_stride, (long long)cols, out)                 \
       : launch_pdl(neb::argmax_kernel<TT, false>, dim3((unsigned)rows), dim3(threads), 0, st, 1,             \
                    static_cast<const TT*>(logits), (long long)row_stride, (long long)cols, out))
  if (dtype == FML_F32) ARGMAX_LAUNCH(float);
  else if (dtype == FML_BF16) ARGMAX_LAUNCH(__nv_bfloat16);
  else ARGMAX_LAUNCH(__half);
#undef ARGMAX_LAUNCH
  count_launch();
  return check_cuda(cudaGetLastError(), "neb_argmax launch");
}

extern "C" int neb_add(const void* a, const void* b, void* y, int64_t n, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "neb_add: bad dtype");
  if (!a || !b || !y || n <= 0) return fail(FML_EINVAL, "neb_add: bad arguments");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = neb::grid_for(n, 256);
  if (dtype == FML_F32)
    launch_pdl(neb::add_kernel<float>, dim3(grid), dim3(256), 0, st, 1, static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(y), n);
  else if (dtype == FML_BF16)
    launch_pdl(neb::add_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, 1, static_cast<const __nv_bfloat16*>(a),
        static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(y), n);
  else
    launch_pdl(neb::add_kernel<__half>, dim3(grid), dim3(256), 0, st, 1, static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<__half*>(y), n);
  count_launch();
  return check_cuda(cudaGetLastError(), "neb_add launch");
}
