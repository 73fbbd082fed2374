// Weighted combine of the k expert outputs plus the gated shared expert (a11).
#include "sg_common.cuh"

namespace sg {

// One thread per 8 consecutive hidden values of one token (16-byte loads).
__global__ void __launch_bounds__(256)
combine_kernel(const uint16_t* __restrict__ y, const uint16_t* __restrict__ scores, int T, int k, int H,
               const uint16_t* __restrict__ shared_y, const uint16_t* __restrict__ shared_gate,
               uint16_t* __restrict__ out) {
  const int vec_per_row = H >> 3;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)T * vec_per_row) return;
  const int t = static_cast<int>(idx / vec_per_row);
  const int v = static_cast<int>(idx - (long long)t * vec_per_row);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int j = 0; j < k; ++j) {
    const float s = bf16_to_f32(scores[(size_t)t * k + j]);
    const uint4 yv = reinterpret_cast<const uint4*>(y + ((size_t)t * k + j) * H)[v];
    const uint32_t w[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] = __fadd_rn(acc[2 * q], round_bf16(__fmul_rn(lo_bf16(w[q]), s)));
      acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], round_bf16(__fmul_rn(hi_bf16(w[q]), s)));
    }
  }
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = round_bf16(acc[i]);
  if (shared_y != nullptr) {
    const float gate = round_bf16(sigmoidf_(bf16_to_f32(shared_gate[t])));
    const uint4 sv = reinterpret_cast<const uint4*>(shared_y + (size_t)t * H)[v];
    const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      o[2 * q] = __fadd_rn(o[2 * q], round_bf16(__fmul_rn(gate, lo_bf16(w[q]))));
      o[2 * q + 1] = __fadd_rn(o[2 * q + 1], round_bf16(__fmul_rn(gate, hi_bf16(w[q]))));
    }
  }
  uint4 r;
  uint32_t* rp = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    rp[q] = static_cast<uint32_t>(f32_to_bf16(o[2 * q])) | (static_cast<uint32_t>(f32_to_bf16(o[2 * q + 1])) << 16);
  reinterpret_cast<uint4*>(out + (size_t)t * H)[v] = r;
}

}  // namespace sg

extern "C" int sg_combine(const uint16_t* y, const uint16_t* scores, int T, int k, int H, const uint16_t* shared_y,
                          const uint16_t* shared_gate, uint16_t* out, void* stream) {
  if (T < 0 || k < 1) return SG_ERR_INVALID_ARG;
  if ((shared_y == nullptr) != (shared_gate == nullptr)) return SG_ERR_INVALID_ARG;
  if (H < 8 || H % 8) return SG_ERR_SHAPE;
  if (T == 0) return SG_OK;
  if (!y || !scores || !out) return SG_ERR_INVALID_ARG;
  const long long n = (long long)T * (H / 8);
  const int threads = 256;
  const long long blocks = (n + threads - 1) / threads;
  if (blocks > 0x7FFFFFFFLL) return SG_ERR_SHAPE;
  sg::combine_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(y, scores, T, k, H, shared_y,
                                                                              shared_gate, out);
  SG_LAUNCH_CHECK();
  return SG_OK;
}
