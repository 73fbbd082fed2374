// Host-side entry points: status text, version, expert byte sizes and the slot
// refill (a8) from a pinned host blob into the arena.
#include <cstring>

#include "sg_common.cuh"

namespace sg {

// Byte size of each of the 9 (or 3) tensors of one expert, in blob order:
// gate, up, down x (weight[, scales, biases]).
static int tensor_sizes(const sg_arena* A, size_t* sz) {
  const size_t H = A->hidden, I = A->inter;
  const size_t n = H * I;
  if (A->bits == 16) {
    sz[0] = sz[1] = sz[2] = n * 2;
    return 3;
  }
  const size_t w = n * A->bits / 8;
  const size_t sb = n / A->group_size * 2;
  for (int p = 0; p < 3; ++p) {
    sz[3 * p] = w;
    sz[3 * p + 1] = sb;
    sz[3 * p + 2] = sb;
  }
  return 9;
}

}  // namespace sg

extern "C" const char* sg_status_string(int status) {
  switch (status) {
    case SG_OK: return "ok";
    case SG_ERR_INVALID_ARG: return "invalid argument (null pointer or negative size)";
    case SG_ERR_SHAPE: return "unsupported shape";
    case SG_ERR_FORMAT: return "unsupported weight format (bits must be 16, 8 or 4; affine group size 64)";
    case SG_ERR_CUDA: return "CUDA runtime error";
    case SG_ERR_CAPACITY: return "caller buffer too small";
    case SG_ERR_TIMEOUT: return "bounded wait expired";
    default: return "unknown status";
  }
}

extern "C" int sg_version(void) { return SG_VERSION; }

extern "C" int sg_built_arch(void) {
#ifdef SG_BUILT_ARCH
  return SG_BUILT_ARCH;
#else
  return 0;
#endif
}

extern "C" size_t sg_expert_bytes(const sg_arena* A) {
  if (!A || (A->bits != 16 && A->bits != 8 && A->bits != 4)) return 0;
  if (A->bits != 16 && A->group_size <= 0) return 0;
  size_t sz[9];
  const int n = sg::tensor_sizes(A, sz);
  size_t tot = 0;
  for (int i = 0; i < n; ++i) tot += sz[i];
  return tot;
}

extern "C" int sg_refill_h2d(const void* blob, size_t blob_len, const sg_arena* A, int sid, void* stream) {
  if (!blob || !A) return SG_ERR_INVALID_ARG;
  if (A->bits != 16 && A->bits != 8 && A->bits != 4) return SG_ERR_FORMAT;
  if (A->bits != 16 && A->group_size != 64) return SG_ERR_FORMAT;
  if (sid < 0 || sid >= A->num_slots) return SG_ERR_SHAPE;
  if (blob_len != sg_expert_bytes(A)) return SG_ERR_SHAPE;
  size_t sz[9];
  const int n = sg::tensor_sizes(A, sz);
  void* dst_base[9];
  if (n == 3) {
    const void* d[3] = {A->gate_w, A->up_w, A->down_w};
    for (int i = 0; i < 3; ++i) dst_base[i] = const_cast<void*>(d[i]);
  } else {
    const void* d[9] = {A->gate_w, A->gate_s, A->gate_b, A->up_w, A->up_s, A->up_b, A->down_w, A->down_s, A->down_b};
    for (int i = 0; i < 9; ++i) dst_base[i] = const_cast<void*>(d[i]);
  }
  for (int i = 0; i < n; ++i)
    if (!dst_base[i]) return SG_ERR_INVALID_ARG;
  const uint8_t* src = static_cast<const uint8_t*>(blob);
  cudaStream_t s = (cudaStream_t)stream;
  for (int i = 0; i < n; ++i) {
    uint8_t* dst = static_cast<uint8_t*>(dst_base[i]) + (size_t)sid * sz[i];
    SG_CUDA_TRY(cudaMemcpyAsync(dst, src, sz[i], cudaMemcpyHostToDevice, s));
    src += sz[i];
  }
  return SG_OK;
}

extern "C" int sg_host_device_ptr(void* host, void** device) {
  if (!host || !device) return SG_ERR_INVALID_ARG;
  void* d = nullptr;
  SG_CUDA_TRY(cudaHostGetDevicePointer(&d, host, 0));
  *device = d;
  return SG_OK;
}
