// Symmetric NVLink peer buffer of the tensor-parallel SUM all-reduce: one per
// TP rank, opened by every peer through CUDA IPC (allreduce.cu), and read and
// written by three kinds of kernel:
//
//   * the standalone all-reduce (allreduce.cu), which splits a message into
//     kArBlocks fixed chunks, one per CTA index;
//   * the GEMM epilogue of the fused decode linear (gemm.cu), which exchanges
//     16-feature sub-blocks of a [features x 32 tokens] partial;
//   * the low-latency (LL) all-reduce (allreduce.cu), whose data words carry
//     their epoch: [2 sets][world slots][2 * slot_bytes] of 8-byte
//     (4 data bytes, 4 epoch bytes) pairs, plus kArBlocks epochs;
//   * the two-shot LL all-reduce (allreduce.cu): a reduce-scatter area like
//     the LL one, an all-gather area [2 sets][2 * slot_bytes] (each position
//     has one writer, its owner rank), plus kArBlocks epochs.
//
// Each kind owns its own data slots, flags and epochs, so they never
// share a buffer region or an epoch counter.  Per flag region, data is
// [2 sets][world slots][slot_bytes], flags [2 sets][world sources][units]
// (u32 epochs raised by the source rank), epochs [units] (this rank's count
// of completed exchanges per unit).
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
  int nsub;              // sub-blocks of the fused region (slot_bytes / 1024)

  __host__ __device__ long long region_bytes(int units) const {
    return 2LL * world * slot_bytes + 2LL * world * units * 4 + (long long)units * 4;
  }
  // region 0: standalone all-reduce; region 1: fused GEMM exchange
  __host__ __device__ long long base(int region) const { return region == 0 ? 0 : region_bytes(kArBlocks); }
  __host__ __device__ int units(int region) const { return region == 0 ? kArBlocks : nsub; }
  __host__ __device__ long long data_off(int region, int set, int slot) const {
    return base(region) + ((long long)set * world + slot) * slot_bytes;
  }
  __host__ __device__ long long flag_off(int region, int set, int src, int unit) const {
    return base(region) + 2LL * world * slot_bytes + (((long long)set * world + src) * units(region) + unit) * 4;
  }
  __host__ __device__ long long epoch_off(int region, int unit) const {
    return base(region) + 2LL * world * slot_bytes + 2LL * world * units(region) * 4 + (long long)unit * 4;
  }
  // region 2: LL all-reduce
  __host__ __device__ long long ll_base() const { return region_bytes(kArBlocks) + region_bytes(nsub); }
  __host__ __device__ long long ll_data_off(int set, int slot) const {
    return ll_base() + ((long long)set * world + slot) * 2 * slot_bytes;
  }
  __host__ __device__ long long ll_epoch_off(int unit) const {
    return ll_base() + 2LL * world * 2 * slot_bytes + (long long)unit * 4;
  }
  // region 3: two-shot LL all-reduce
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
