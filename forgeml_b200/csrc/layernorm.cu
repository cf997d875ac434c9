// LayerNorm over the trailing dimension (warp per row, fp32 statistics).
//
// Replaces F.layer_norm as evaluated by the reference in
// src/forgeml/ops.py:54-60 (ForgeML layer_norm nodes) and
// src/nebula/runtime.py:130,151,185 (Nebula pre-LN and final norm).
//
//   y = (x - mean) / sqrt(var + eps) * gamma + beta,  var biased (1/cols),
//
// computed in fp32 with an exact two-pass mean/variance and one rounding to
// the output dtype.  HBM-bound: each element is read once (the row is cached
// in registers between passes) and written once; 16-byte vector accesses.
#include <string>

#include "common.cuh"

namespace fml {
namespace ln {

constexpr int kWarps = 4;

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* in) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(in[i]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Vectorised path: cols = 32 * VPL_MAX-or-fewer vectors per lane, 16-byte
// aligned rows.  The row lives in registers between the passes.
template <typename T, int VPL_MAX>
__global__ void __launch_bounds__(kWarps * 32)
    ln_vec_kernel(const T* __restrict__ x, long long xs, const T* __restrict__ g,
                  const T* __restrict__ b, float eps, T* __restrict__ y, long long ys, long long rows,
                  int cols) {
  constexpr int W = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int nvec = cols / W;
  // gamma / beta are constant weights: this lane's vectors are loaded into
  // registers while the previous grid finishes, off the row's dependency
  // chain (rows up to 8 vectors per lane; wider rows prefetch them to L2).
  constexpr bool kPreload = VPL_MAX <= 8;
  uint4 graw[kPreload ? VPL_MAX : 1], braw[kPreload ? VPL_MAX : 1];
  if (g != nullptr) {
#pragma unroll
    for (int i = 0; i < VPL_MAX; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        if constexpr (kPreload) {
          graw[i] = *reinterpret_cast<const uint4*>(g + vi * W);
          braw[i] = *reinterpret_cast<const uint4*>(b + vi * W);
        } else if ((vi & 7) == 0) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(g + vi * W));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(b + vi * W));
        }
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  const long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const T* xr = x + row * xs;
  float v[VPL_MAX][W];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL_MAX; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      load_vec<T>(xr + vi * W, v[i]);
#pragma unroll
      for (int e = 0; e < W; ++e) sum += v[i][e];
    }
  }
  const float mean = warp_sum(sum) / (float)cols;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL_MAX; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < W; ++e) {
        const float d = v[i][e] - mean;
        sq += d * d;
      }
    }
  }
  const float var = warp_sum(sq) / (float)cols;
  const float rstd = 1.0f / sqrtf(var + eps);
  T* yr = y + row * ys;
#pragma unroll
  for (int i = 0; i < VPL_MAX; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      float o[W];
      float gv[W], bv[W];
      if (g != nullptr) {
        if constexpr (kPreload) {
          const T* ge = reinterpret_cast<const T*>(&graw[i]);
          const T* be = reinterpret_cast<const T*>(&braw[i]);
#pragma unroll
          for (int e = 0; e < W; ++e) {
            gv[e] = to_f32<T>(ge[e]);
            bv[e] = to_f32<T>(be[e]);
          }
        } else {
          load_vec<T>(g + vi * W, gv);
          load_vec<T>(b + vi * W, bv);
        }
      }
#pragma unroll
      for (int e = 0; e < W; ++e) {
        float t = (v[i][e] - mean) * rstd;
        if (g != nullptr) t = t * gv[e] + bv[e];
        o[e] = t;
      }
      store_vec<T>(yr + vi * W, o);
    }
  }
}

// General path (any cols / alignment): three passes over the row, the later
// ones served from L1/L2.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    ln_generic_kernel(const T* __restrict__ x, long long xs, const T* __restrict__ g,
                      const T* __restrict__ b, float eps, T* __restrict__ y, long long ys,
                      long long rows, int cols) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const T* xr = x + row * xs;
  float sum = 0.f;
  for (int c = lane; c < cols; c += 32) sum += to_f32<T>(xr[c]);
  const float mean = warp_sum(sum) / (float)cols;
  float sq = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float d = to_f32<T>(xr[c]) - mean;
    sq += d * d;
  }
  const float var = warp_sum(sq) / (float)cols;
  const float rstd = 1.0f / sqrtf(var + eps);
  T* yr = y + row * ys;
  for (int c = lane; c < cols; c += 32) {
    float t = (to_f32<T>(xr[c]) - mean) * rstd;
    if (g != nullptr) t = t * to_f32<T>(g[c]) + to_f32<T>(b[c]);
    yr[c] = from_f32<T>(t);
  }
}

template <typename T>
static int launch(const void* x, long long xs, const void* g, const void* b, float eps, void* y,
                  long long ys, long long rows, long long cols, cudaStream_t st) {
  constexpr int W = Vec<T>::N;
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  const bool aligned = (cols % W == 0) && (xs % W == 0) && (ys % W == 0) &&
                       (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                       (g == nullptr || (reinterpret_cast<uintptr_t>(g) % 16 == 0 &&
                                         reinterpret_cast<uintptr_t>(b) % 16 == 0));
  const long long vpl = (cols / W + 31) / 32;
  const T* xp = static_cast<const T*>(x);
  const T* gp = static_cast<const T*>(g);
  const T* bp = static_cast<const T*>(b);
  T* yp = static_cast<T*>(y);
  if (aligned && vpl <= 2)
    launch_pdl(ln_vec_kernel<T, 2>, dim3(grid), dim3(kWarps * 32), 0, st, 1, xp, xs, gp, bp, eps, yp, ys, rows, (int)cols);
  else if (aligned && vpl <= 4)
    launch_pdl(ln_vec_kernel<T, 4>, dim3(grid), dim3(kWarps * 32), 0, st, 1, xp, xs, gp, bp, eps, yp, ys, rows, (int)cols);
  else if (aligned && vpl <= 8)
    launch_pdl(ln_vec_kernel<T, 8>, dim3(grid), dim3(kWarps * 32), 0, st, 1, xp, xs, gp, bp, eps, yp, ys, rows, (int)cols);
  else if (aligned && vpl <= 16)
    launch_pdl(ln_vec_kernel<T, 16>, dim3(grid), dim3(kWarps * 32), 0, st, 1, xp, xs, gp, bp, eps, yp, ys, rows, (int)cols);
  else
    launch_pdl(ln_generic_kernel<T>, dim3(grid), dim3(kWarps * 32), 0, st, 1, xp, xs, gp, bp, eps, yp, ys, rows, (int)cols);
  count_launch();
  return check_cuda(cudaGetLastError(), "layernorm launch");
}

}  // namespace ln
}  // namespace fml

using namespace fml;

extern "C" int fml_layernorm(const void* x, int64_t x_row_stride, const void* gamma,
                             const void* beta, float eps, void* y, int64_t y_row_stride,
                             int64_t rows, int64_t cols, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(FML_EINVAL, "layernorm: bad dtype");
  if (!x || !y) return fail(FML_EINVAL, "layernorm: null pointer");
  if (rows <= 0 || cols <= 0) return fail(FML_EINVAL, "layernorm: rows and cols must be positive");
  if (cols > (1 << 30)) return fail(FML_EUNSUPPORTED, "layernorm: cols too large");
  if ((gamma == nullptr) != (beta == nullptr))
    return fail(FML_EINVAL, "layernorm: gamma and beta must be given together");
  if (!(eps > 0.f)) return fail(FML_EINVAL, "layernorm: eps must be positive");
  if (x_row_stride < cols || y_row_stride < cols)
    return fail(FML_EINVAL, "layernorm: row stride smaller than cols");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FML_F32)
    return ln::launch<float>(x, x_row_stride, gamma, beta, eps, y, y_row_stride, rows, cols, st);
  if (dtype == FML_BF16)
    return ln::launch<__nv_bfloat16>(x, x_row_stride, gamma, beta, eps, y, y_row_stride, rows,
                                     cols, st);
  return ln::launch<__half>(x, x_row_stride, gamma, beta, eps, y, y_row_stride, rows, cols, st);
}
