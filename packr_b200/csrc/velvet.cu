// Per-parameter means of the int8 second-moment state, for VelvetController
// (reference packr/velvet.py:270-300 computes one `.item()` per parameter).
// One launch covers every parameter: CTAs (chunk, parameter) each add up a
// 64K-element chunk in double and fold it into the parameter's slot with one
// atomic add per warp; the host reads all slots with a single copy.
//   scaled   (block_size > 0):  sum_i v[i] * v_scale[(block_origin + i) / block_size]
//   unscaled (block_size == 0): sum_i v[i]
// A whole parameter's state uses origin 0 (the reference's mean over the
// [blocks, block_size] view; unscaled when that view would need padding); a
// parameter's slice of a data-parallel flat shard passes its offset into the
// shard's block grid.  The host divides by numel.
#include "common.cuh"

namespace packr {
namespace velvet {

constexpr int kThreads = 256;
constexpr long long kChunk = 65536;

struct Desc {
  const int8_t* v;
  const float* v_scale;
  long long numel;
  long long block_size;  // 0: unscaled
  long long block_origin;
};

constexpr int kMaxDescs = 512;
struct Launch {
  int n;
  Desc d[kMaxDescs];
};

__global__ void __launch_bounds__(kThreads) v_sums_kernel(const __grid_constant__ Launch L, double* __restrict__ sums) {
  const Desc& d = L.d[blockIdx.y];
  const long long c0 = (long long)blockIdx.x * kChunk;
  if (c0 >= d.numel) return;
  const long long c1 = c0 + kChunk < d.numel ? c0 + kChunk : d.numel;
  double s = 0.0;
  for (long long i = c0 + threadIdx.x; i < c1; i += kThreads) {
    const double code = (double)d.v[i];
    s += d.block_size > 0 ? code * (double)__ldg(d.v_scale + (d.block_origin + i) / d.block_size) : code;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(sums + blockIdx.y, s);
}

}  // namespace velvet
}  // namespace packr

extern "C" int packr_state_v_sums(const packr_vsum_desc* descs, int n, double* sums, void* stream) {
  using namespace packr;
  if (n < 0 || (n > 0 && (descs == nullptr || sums == nullptr))) return PACKR_ERR_INVALID_ARGUMENT;
  if (n == 0) return PACKR_OK;
  if (!aligned(sums, 8)) return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(sums, 0, (size_t)n * sizeof(double), s) != cudaSuccess) return PACKR_ERR_CUDA;
  for (int base = 0; base < n; base += velvet::kMaxDescs) {
    velvet::Launch L;
    L.n = n - base < velvet::kMaxDescs ? n - base : velvet::kMaxDescs;
    long long max_chunks = 1;
    for (int i = 0; i < L.n; ++i) {
      const packr_vsum_desc& d = descs[base + i];
      if (d.numel < 0 || d.block_size < 0 || d.block_origin < 0) return PACKR_ERR_SHAPE;
      if (d.numel > 0 && d.v == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
      if (d.block_size > 0 && d.v_scale == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
      L.d[i] = {d.v, d.v_scale, d.numel, d.block_size, d.block_origin};
      const long long c = (d.numel + velvet::kChunk - 1) / velvet::kChunk;
      if (c > max_chunks) max_chunks = c;
    }
    if (max_chunks > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
    velvet::v_sums_kernel<<<dim3((unsigned)max_chunks, (unsigned)L.n), velvet::kThreads, 0, s>>>(L, sums + base);
    if ((st = launch_status()) != PACKR_OK) return st;
  }
  return PACKR_OK;
}
