// Symmetric NVLink peer buffer of the tensor-parallel SUM all-reduce: one per
// TP rank, opened by every peer through CUDA IPC (allreduce.cu), and read and
// written by three kinds of kernel, each in a region of its own:
//
//   * exchange: the all-reduce fused into the decode GEMM's epilogue
//     (gemm.cu), which exchanges 16-feature sub-blocks of a [features x 32
//     tokens] partial: data [2 sets][world slots][slot_bytes], flags
//     [2 sets][world sources][nsub] (u32 epochs raised by the source rank),
//     epochs [nsub] (this rank's count of completed exchanges per sub-block);
//   * ll: the one-shot low-latency all-reduce (allreduce.cu), whose data words
//     carry their epoch: [2 sets][world slots][2 * slot_bytes] of 8-byte
//     (4 data bytes, 4 epoch bytes) pairs, plus kArBlocks epochs;
//   * ts: the two-shot LL all-reduce (allreduce.cu): a reduce-scatter area
//     like the LL one, an all-gather area [2 sets][2 * slot_bytes] (each
//     position has one writer, its owner rank), plus kArBlocks epochs.
//
// No two kinds share a byte or an epoch counter.
#pragma once

#include <stdint.h>

namespace fml {
namespace peer {

constexpr int kMaxWorld = 8;
constexpr int kArBlocks = 128;     // chunks (and CTAs) of the standalone all-reduce
constexpr int kSubFeatures = 16;   // features per sub-block of the fused exchange
constexpr int kSubTokens = 32;     // token capacity of a sub-block (the decode GEMM's BN)

struct Layout {
  long long slot_bytes;  // one rank's message, per region
  int world;
  int nsub;              // sub-blocks of the exchange region (slot_bytes / 1 KB)

  // exchange region, at offset 0
  __host__ __device__ long long ex_data_off(int set, int slot) const {
    return ((long long)set * world + slot) * slot_bytes;
  }
  __host__ __device__ long long ex_flag_off(int set, int src, int unit) const {
    return 2LL * world * slot_bytes + (((long long)set * world + src) * nsub + unit) * 4;
  }
  __host__ __device__ long long ex_epoch_off(int unit) const {
    return 2LL * world * slot_bytes + 2LL * world * nsub * 4 + (long long)unit * 4;
  }
  __host__ __device__ long long ex_bytes() const {
    return 2LL * world * slot_bytes + 2LL * world * nsub * 4 + (long long)nsub * 4;
  }
  // ll region
  __host__ __device__ long long ll_base() const { return (ex_bytes() + 15) / 16 * 16; }
  __host__ __device__ long long ll_data_off(int set, int slot) const {
    return ll_base() + ((long long)set * world + slot) * 2 * slot_bytes;
  }
  __host__ __device__ long long ll_epoch_off(int unit) const {
    return ll_base() + 2LL * world * 2 * slot_bytes + (long long)unit * 4;
  }
  // ts region
  __host__ __device__ long long ts_base() const { return ll_base() + 4LL * world * slot_bytes + kArBlocks * 4; }
  __host__ __device__ long long ts_rs_off(int set, int slot) const {
    return ts_base() + ((long long)set * world + slot) * 2 * slot_bytes;
  }
  __host__ __device__ long long ts_ag_off(int set) const {
    return ts_base() + 4LL * world * slot_bytes + (long long)set * 2 * slot_bytes;
  }
  __host__ __device__ long long ts_epoch_off(int unit) const {
    return ts_base() + 4LL * world * slot_bytes + 4LL * slot_bytes + (long long)unit * 4;
  }
  __host__ __device__ long long total() const {
    return ts_base() + 4LL * world * slot_bytes + 4LL * slot_bytes + kArBlocks * 4;
  }
};

// What a kernel needs to reach every rank's buffer.
struct View {
  uint8_t* base[kMaxWorld];  // every rank's buffer mapped into this process (own included)
  Layout lay;
  int rank;
  long long timeout_cycles;
};

// Host object behind the neb_ar_* handle.
struct Ctx {
  View v;
  uint8_t* own = nullptr;
  bool opened[kMaxWorld] = {};
  int device = 0;
  int proto = 0;  // standalone all-reduce: 0 by group size, 1 one-shot LL, 2 two-shot LL
};

#ifdef __CUDACC__
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
#endif

}  // namespace peer
}  // namespace fml
