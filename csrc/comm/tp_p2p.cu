// Tensor-parallel (sequence-parallel) row collectives over NVLink peer memory (sm_100a).
//
// The reference only models these collectives (perf_model/scaling.py:151-153: four per layer
// as ring all-reduces). Under sequence parallelism each rank of a tensor-parallel group owns
// rows [r n, (r+1) n) of the N = tp n token rows. Every rank's buffers are CUDA-IPC mapped into
// every other rank, so a kernel moves rows with plain 16-byte loads and stores through
// NVSwitch (no multicast, no NCCL):
//   all-gather     each rank stores its n rows into every peer's (N, d) buffer
//   reduce-scatter each rank stores row r of its (N, d) partial into slot `rank` of row r's
//                  owner; the owner sums its tp slots (the GEMM producing the partial can do the
//                  stores itself: the PEER_RS epilogue of csrc/gemm)
// Completion across ranks is the flag barrier of csrc/comm/dp_fused.cu (bounded waits).
#include "../common/common.cuh"

namespace llmt {
namespace {

constexpr int kMaxTp = 8;

__global__ void __launch_bounds__(256) allgather_rows_kernel(const uint4* __restrict__ src, void* const* dst, int tp,
                                                             int64_t off16, int64_t n16) {
  uint4* d[kMaxTp];
#pragma unroll
  for (int p = 0; p < kMaxTp; ++p) d[p] = p < tp ? reinterpret_cast<uint4*>(dst[p]) + off16 : nullptr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = __ldg(src + i);
#pragma unroll
    for (int p = 0; p < kMaxTp; ++p)
      if (p < tp) __stcg(d[p] + i, v);
  }
  __threadfence_system();
}

// Row r of the (N, d) partial -> slot `rank` of owner q = r / n: (rank * n + r - q n) * d.
__global__ void __launch_bounds__(256) scatter_rows_kernel(const uint4* __restrict__ src, void* const* slots,
                                                           int rank, int64_t n, int d16, int64_t total16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total16;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / d16;
    const int c = (int)(i - r * d16);
    const int64_t q = r / n;
    // every slot buffer holds tp * n rows: the same extent as the source
    if (!LLMT_IN(((int64_t)rank * n + (r - q * n)) * d16 + c, ((int64_t)rank * n + (r - q * n)) * d16 + c + 1,
                 total16, 501))
      continue;
    uint4* dst = reinterpret_cast<uint4*>(slots[q]) + ((int64_t)rank * n + (r - q * n)) * d16 + c;
    __stcg(dst, __ldg(src + i));
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) sum_slots_kernel(const uint4* __restrict__ slots, uint4* __restrict__ out,
                                                        int tp, int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < tp; ++p) {
      // slots were written by peers through NVLink before the barrier: read around L1
      const uint4 v = __ldcg(slots + (int64_t)p * n16 + i);
      float f[8];
      bf16x8_to_float(*reinterpret_cast<const BF16x8*>(&v), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    const BF16x8 o = float_to_bf16x8(acc);
    out[i] = *reinterpret_cast<const uint4*>(&o);
  }
}

inline int grid_for(int64_t n16) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n16, 256), (int64_t)sm_count() * 8));
}

}  // namespace

cudaError_t tp_allgather_rows(const void* src, void* const* dst, int tp, int64_t row0, int64_t rows, int d,
                              cudaStream_t st) {
  LLMT_REQUIRE(tp >= 1 && tp <= kMaxTp, "tp_allgather_rows: 1 <= tp <= 8");
  LLMT_REQUIRE(d % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0, "tp_allgather_rows: 16-byte rows");
  const int64_t n16 = rows * d / 8;
  if (n16 == 0) return cudaSuccess;
  allgather_rows_kernel<<<grid_for(n16), 256, 0, st>>>(static_cast<const uint4*>(src), dst, tp, row0 * d / 8, n16);
  return cudaGetLastError();
}

cudaError_t tp_scatter_rows(const void* src, void* const* slots, int tp, int rank, int64_t rows_per_rank, int d,
                            cudaStream_t st) {
  LLMT_REQUIRE(tp >= 1 && tp <= kMaxTp && rank >= 0 && rank < tp, "tp_scatter_rows: rank / tp");
  LLMT_REQUIRE(d % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0, "tp_scatter_rows: 16-byte rows");
  const int64_t total16 = (int64_t)tp * rows_per_rank * d / 8;
  if (total16 == 0) return cudaSuccess;
  scatter_rows_kernel<<<grid_for(total16), 256, 0, st>>>(static_cast<const uint4*>(src), slots, rank, rows_per_rank,
                                                         d / 8, total16);
  return cudaGetLastError();
}

cudaError_t tp_sum_slots(const void* slots, void* out, int tp, int64_t rows, int d, cudaStream_t st) {
  LLMT_REQUIRE(tp >= 1 && tp <= kMaxTp && d % 8 == 0, "tp_sum_slots: tp / width");
  const int64_t n16 = rows * d / 8;
  if (n16 == 0) return cudaSuccess;
  sum_slots_kernel<<<grid_for(n16), 256, 0, st>>>(static_cast<const uint4*>(slots), static_cast<uint4*>(out), tp, n16);
  return cudaGetLastError();
}

}  // namespace llmt
