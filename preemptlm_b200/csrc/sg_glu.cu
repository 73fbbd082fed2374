// Gathered SwiGLU expert matmuls over the slot arena (a9, a10, a12):
// streaming GEMV-style kernels for decode batch sizes.
//
// Work item = (group u, block of output rows).  A group is one expert slot with
// the pairs routed to it (sg_dispatch layout).  Eight warps per CTA; each warp
// owns WROWS weight rows and splits K across lanes in chunks of 16 weights
// (lane j takes chunks j, j+32, ...).  The pairs' input rows are staged in
// shared memory NT at a time.  Affine weights are never expanded: per chunk a
// lane forms dot = sum(q * x) and xs = sum(x) and adds scale*dot + bias*xs,
// which equals sum((scale*q + bias) * x) without the bf16 rounding of w.
#include <mutex>

#include "sg_common.cuh"

namespace sg {

constexpr int GW_WARPS = 8;
constexpr int GW_NT = 8;      // pairs staged per pass
constexpr int GW_CHUNK = 16;  // weights per lane step

// --------------------------------------------------------------- weight chunk
template <int BITS>
struct Chunk;

template <>
struct Chunk<16> {  // 16 bf16 = 32 bytes
  uint4 a, b;
  __device__ __forceinline__ void load(const uint8_t* row, int c) {
    const uint4* p = reinterpret_cast<const uint4*>(row + (size_t)c * 32);
    a = ldg_nc_v4(p);
    b = ldg_nc_v4(p + 1);
  }
  __device__ __forceinline__ void to_float(float* w) const {
    const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[2 * i] = lo_bf16(v[i]);
      w[2 * i + 1] = hi_bf16(v[i]);
    }
  }
};

__device__ __forceinline__ float u8f(uint32_t q) {  // exact small unsigned int -> fp32
  return __fsub_rn(__uint_as_float(0x4B000000u | q), 8388608.0f);
}

template <>
struct Chunk<8> {  // 16 x u8 = 16 bytes
  uint4 a;
  __device__ __forceinline__ void load(const uint8_t* row, int c) {
    a = ldg_nc_v4(row + (size_t)c * 16);
  }
  __device__ __forceinline__ void to_float(float* w) const {
    const uint32_t v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int m = 0; m < 4; ++m) w[4 * i + m] = u8f((v[i] >> (8 * m)) & 0xFFu);
  }
};

template <>
struct Chunk<4> {  // 16 x u4 = 8 bytes
  uint2 a;
  __device__ __forceinline__ void load(const uint8_t* row, int c) {
    a = __ldg(reinterpret_cast<const uint2*>(row + (size_t)c * 8));
  }
  __device__ __forceinline__ void to_float(float* w) const {
    const uint32_t v[2] = {a.x, a.y};
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int m = 0; m < 8; ++m) w[8 * i + m] = u8f((v[i] >> (4 * m)) & 0xFu);
  }
};

struct Mat {  // one projection of the arena
  const uint8_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int out, k;
};

__device__ __forceinline__ size_t row_bytes(int bits, int k) { return (size_t)k * bits / 8; }

// Accumulate WROWS rows x NT pairs over the whole K range.
template <int BITS, int WROWS, int NT>
__device__ __forceinline__ void gemv_rows(const Mat* mats, const int* mrow, int slot, const uint16_t* xs_smem, int K,
                                          float (&acc)[WROWS][GW_NT]) {
  const int lane = threadIdx.x & 31;
  const int nchunks = K / GW_CHUNK;
  const int groups = K / 64;
  for (int c = lane; c < nchunks; c += 32) {
    Chunk<BITS> ch[WROWS];
    float sc[WROWS], bi[WROWS];
#pragma unroll
    for (int a = 0; a < WROWS; ++a) {
      const Mat& m = mats[a];
      const size_t r = (size_t)slot * m.out + mrow[a];
      ch[a].load(m.w + r * row_bytes(BITS, K), c);
      if (BITS != 16) {
        sc[a] = bf16_to_f32(__ldg(m.s + r * groups + (c >> 2)));
        bi[a] = bf16_to_f32(__ldg(m.b + r * groups + (c >> 2)));
      }
    }
#pragma unroll
    for (int b = 0; b < NT; ++b) {
      const uint4* xp = reinterpret_cast<const uint4*>(xs_smem + (size_t)b * K + (size_t)c * GW_CHUNK);
      const uint4 x0 = xp[0], x1 = xp[1];
      const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      float xf[16];
      float xsum = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xf[2 * i] = lo_bf16(xv[i]);
        xf[2 * i + 1] = hi_bf16(xv[i]);
      }
      if (BITS != 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) xsum += xf[i];
      }
#pragma unroll
      for (int a = 0; a < WROWS; ++a) {
        float wf[16];
        ch[a].to_float(wf);
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) dot = fmaf(wf[i], xf[i], dot);
        if (BITS != 16) {
          acc[a][b] = fmaf(sc[a], dot, acc[a][b]);
          acc[a][b] = fmaf(bi[a], xsum, acc[a][b]);
        } else {
          acc[a][b] += dot;
        }
      }
    }
  }
}

// DUAL: gate/up fused with SwiGLU -> h[p, I];  !DUAL: down -> y[p, H].
template <int BITS, bool DUAL>
__global__ void __launch_bounds__(GW_WARPS * 32)
gemv_glu_kernel(sg_arena A, const uint16_t* __restrict__ xin, int pair_div, const int32_t* __restrict__ counts,
                const int32_t* __restrict__ slot_ids, const int32_t* __restrict__ group_off,
                const int32_t* __restrict__ perm, uint16_t* __restrict__ out, int in_by_pos, int out_by_pos) {
  constexpr int WROWS = 4;                        // weight rows per warp
  constexpr int OROWS = DUAL ? WROWS / 2 : WROWS;  // output rows per warp
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);  // [GW_NT][K]
  const int u = blockIdx.y;
  if (u >= counts[0]) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = A.hidden, I = A.inter;
  const int K = DUAL ? H : I;
  const int OUT = DUAL ? I : H;
  const int orow0 = (blockIdx.x * GW_WARPS + warp) * OROWS;
  const int slot = slot_ids[u];
  const int p_begin = group_off[u], p_end = group_off[u + 1];
  const bool slot_ok = slot >= 0 && slot < A.num_slots;

  Mat mats[WROWS];
  int mrow[WROWS];
#pragma unroll
  for (int a = 0; a < WROWS; ++a) {
    int r = DUAL ? orow0 + (a % OROWS) : orow0 + a;
    mrow[a] = r < OUT ? r : OUT - 1;  // clamp reads; writes are masked
    if (DUAL) {
      const bool g = a < OROWS;
      mats[a] = Mat{static_cast<const uint8_t*>(g ? A.gate_w : A.up_w), static_cast<const uint16_t*>(g ? A.gate_s : A.up_s),
                    static_cast<const uint16_t*>(g ? A.gate_b : A.up_b), I, H};
    } else {
      mats[a] = Mat{static_cast<const uint8_t*>(A.down_w), static_cast<const uint16_t*>(A.down_s),
                    static_cast<const uint16_t*>(A.down_b), H, I};
    }
  }

  for (int p0 = p_begin; p0 < p_end; p0 += GW_NT) {
    const int nb = min(GW_NT, p_end - p0);
    __syncthreads();
    const int cpr = K / 8;  // 16-byte chunks per row
    for (int c = threadIdx.x; c < GW_NT * cpr; c += blockDim.x) {
      int b = c / cpr, cc = c - b * cpr;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (b < nb) {
        int row = in_by_pos ? p0 + b : perm[p0 + b] / pair_div;
        v = reinterpret_cast<const uint4*>(xin + (size_t)row * K)[cc];
      }
      reinterpret_cast<uint4*>(xs)[c] = v;
    }
    __syncthreads();
    float acc[WROWS][GW_NT];
#pragma unroll
    for (int a = 0; a < WROWS; ++a)
#pragma unroll
      for (int b = 0; b < GW_NT; ++b) acc[a][b] = 0.0f;
    if (slot_ok && orow0 < OUT) {
      if (nb == 1) gemv_rows<BITS, WROWS, 1>(mats, mrow, slot, xs, K, acc);
      else if (nb == 2) gemv_rows<BITS, WROWS, 2>(mats, mrow, slot, xs, K, acc);
      else if (nb <= 4) gemv_rows<BITS, WROWS, 4>(mats, mrow, slot, xs, K, acc);
      else gemv_rows<BITS, WROWS, GW_NT>(mats, mrow, slot, xs, K, acc);
    }
    if (orow0 >= OUT) continue;
    // fold partials and write: lane (o * GW_NT + b) owns output row o, pair b
#pragma unroll
    for (int o = 0; o < OROWS; ++o) {
#pragma unroll
      for (int b = 0; b < GW_NT; ++b) {
        if (b >= nb) break;
        const int r = orow0 + o;
        if (DUAL) {
          float g = warp_fold_sum(acc[o][b]);
          float up = warp_fold_sum(acc[o + OROWS][b]);
          if (lane == ((o * GW_NT + b) & 31) && r < OUT) {
            const int p = out_by_pos ? p0 + b : perm[p0 + b];
            out[(size_t)p * OUT + r] = slot_ok ? swiglu_bf16(g, up) : (uint16_t)0;
          }
        } else {
          float y = warp_fold_sum(acc[o][b]);
          if (lane == ((o * GW_NT + b) & 31) && r < OUT) {
            const int p = out_by_pos ? p0 + b : perm[p0 + b];
            out[(size_t)p * OUT + r] = slot_ok ? f32_to_bf16(y) : (uint16_t)0;
          }
        }
      }
    }
  }
}

template <int BITS, bool DUAL>
static int launch_gemv(const sg_arena* A, const uint16_t* xin, int pair_div, const int32_t* counts,
                       const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                       uint16_t* out, int in_by_pos, int out_by_pos, cudaStream_t s) {
  const int K = DUAL ? A->hidden : A->inter;
  const int OUT = DUAL ? A->inter : A->hidden;
  const int orows_cta = GW_WARPS * (DUAL ? 2 : 4);
  const size_t smem = (size_t)GW_NT * K * 2;
  static bool attr_done = false;
  if (!attr_done) {
    SG_CUDA_TRY(cudaFuncSetAttribute(gemv_glu_kernel<BITS, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     160 * 1024));
    attr_done = true;
  }
  dim3 grid((OUT + orows_cta - 1) / orows_cta, grid_groups);
  gemv_glu_kernel<BITS, DUAL><<<grid, GW_WARPS * 32, smem, s>>>(*A, xin, pair_div, counts, slot_ids, group_off,
                                                                 perm, out, in_by_pos, out_by_pos);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

int check_arena(const sg_arena* A) {
  if (!A || !A->gate_w || !A->up_w || !A->down_w) return SG_ERR_INVALID_ARG;
  if (A->num_slots < 1 || A->hidden < 64 || A->inter < 64) return SG_ERR_SHAPE;
  if (A->hidden % 64 || A->inter % 64) return SG_ERR_SHAPE;
  if ((size_t)A->hidden * 2 * GW_NT > 160 * 1024 || (size_t)A->inter * 2 * GW_NT > 160 * 1024) return SG_ERR_SHAPE;
  if (A->bits == 16) return SG_OK;
  if (A->bits != 4 && A->bits != 8) return SG_ERR_FORMAT;
  if (A->group_size != 64) return SG_ERR_FORMAT;
  if (!A->gate_s || !A->gate_b || !A->up_s || !A->up_b || !A->down_s || !A->down_b) return SG_ERR_INVALID_ARG;
  return SG_OK;
}

}  // namespace sg

namespace sg {
bool tc_supported(const sg_arena* A, bool dual, int grid_groups);
int tc_glu_launch(const sg_arena* A, bool dual, const uint16_t* in, int in_rows, int pair_div, int in_by_pos,
                  int out_by_pos, int P, const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                  const int32_t* perm, int grid_groups, uint16_t* out, cudaStream_t s);
int tc_dense_launch(const sg_arena* A, bool dual, const uint16_t* in, int rows, int sid, uint16_t* out,
                    cudaStream_t s);
static int g_glu_path = 0;  // 0 auto, 1 streaming GEMV, 2 tcgen05, 3 tcgen05 over permuted rows

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// auto: the tensor-core path once the mean pairs per group reaches 2, or once
// the groups give at least one tile per SM (a tile streams 128 weight rows
// at the HBM rate whatever its pair count, so it beats the CUDA-core GEMV
// from one pair per group on); the GEMV serves the few-expert steps whose
// tiles would leave most SMs idle.
static bool use_tc(const sg_arena* A, bool dual, int P, int grid_groups) {
  if (g_glu_path == 1 || !tc_supported(A, dual, grid_groups)) return false;
  if (g_glu_path >= 2) return true;
  const int out = dual ? A->inter : A->hidden;
  const long long tiles = (long long)grid_groups * (out / 128);
  return P >= 2 * grid_groups || tiles >= sm_count();
}

// Whether sg_glu_forward first copies the pairs' token rows into dispatch
// order: worth it once a group's pairs fill 64-wide tiles (a contiguous
// tile of rows then loads with one TMA box per stage).
static bool use_permute(const sg_arena* A, int P, int grid_groups) {
  if (!use_tc(A, true, P, grid_groups) || !use_tc(A, false, P, grid_groups)) return false;
  if (g_glu_path == 3) return true;
  return P >= 32 * grid_groups;
}

// xs[pos] = x[perm[pos] / pair_div]: one warp per row, 16-byte chunks.
__global__ void __launch_bounds__(256)
permute_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm, int pair_div, int P, int H,
                    uint16_t* __restrict__ xs) {
  const int pos = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= P) return;
  const int row = perm[pos] / pair_div;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)pos * H);
  for (int c = threadIdx.x & 31; c < H / 8; c += 32) dst[c] = ldg_nc_v4(src + c);
}

static int glu_dual(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div, const int32_t* counts,
                    const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                    uint16_t* h, int flags, cudaStream_t s) {
  const int in_pos = (flags & SG_IN_DISPATCH_ORDER) != 0, out_pos = (flags & SG_OUT_DISPATCH_ORDER) != 0;
  const int div = in_pos ? 1 : pair_div;
  if (use_tc(arena, true, num_pairs, grid_groups)) {
    const int in_rows = in_pos ? num_pairs : (num_pairs + pair_div - 1) / pair_div;
    return tc_glu_launch(arena, true, x, in_rows, div, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, h, s);
  }
  switch (arena->bits) {
    case 16: return launch_gemv<16, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, s);
    case 8: return launch_gemv<8, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, s);
    default: return launch_gemv<4, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, s);
  }
}

static int glu_single(const sg_arena* arena, const uint16_t* h, int num_pairs, const int32_t* counts,
                      const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                      uint16_t* y, int flags, cudaStream_t s) {
  const int in_pos = (flags & SG_IN_DISPATCH_ORDER) != 0, out_pos = (flags & SG_OUT_DISPATCH_ORDER) != 0;
  if (use_tc(arena, false, num_pairs, grid_groups))
    return tc_glu_launch(arena, false, h, num_pairs, 1, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, y, s);
  switch (arena->bits) {
    case 16: return launch_gemv<16, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, s);
    case 8: return launch_gemv<8, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, s);
    default: return launch_gemv<4, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, s);
  }
}

static int check_glu_args(const sg_arena* arena, int num_pairs, int pair_div, int grid_groups, int flags) {
  int st = check_arena(arena);
  if (st) return st;
  if (num_pairs < 0 || pair_div < 1 || grid_groups < 0) return SG_ERR_INVALID_ARG;
  if (flags & ~(SG_IN_DISPATCH_ORDER | SG_OUT_DISPATCH_ORDER)) return SG_ERR_INVALID_ARG;
  if (grid_groups > 65535) return SG_ERR_SHAPE;
  return SG_OK;
}
}  // namespace sg

extern "C" int sg_set_glu_path(int mode) {
  if (mode < 0 || mode > 3) return SG_ERR_INVALID_ARG;
  sg::g_glu_path = mode;
  return SG_OK;
}

extern "C" int sg_glu_use_permute(const sg_arena* arena, int num_pairs, int grid_groups) {
  if (sg::check_arena(arena) || num_pairs <= 0 || grid_groups <= 0) return 0;
  return sg::use_permute(arena, num_pairs, grid_groups) ? 1 : 0;
}

extern "C" int sg_permute_rows(const uint16_t* x, const int32_t* perm, int pair_div, int num_pairs, int H,
                               uint16_t* xs, void* stream) {
  if (num_pairs < 0 || pair_div < 1 || H < 8 || H % 8) return num_pairs < 0 || pair_div < 1 ? SG_ERR_INVALID_ARG
                                                                                            : SG_ERR_SHAPE;
  if (num_pairs == 0) return SG_OK;
  if (!x || !perm || !xs) return SG_ERR_INVALID_ARG;
  sg::permute_rows_kernel<<<(num_pairs + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, perm, pair_div, num_pairs, H, xs);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_glu_gate_up(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                              const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                              const int32_t* perm, int grid_groups, uint16_t* h, int flags, void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, flags);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !h) return SG_ERR_INVALID_ARG;
  return sg::glu_dual(arena, x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, h, flags,
                      (cudaStream_t)stream);
}

extern "C" int sg_glu_down(const sg_arena* arena, const uint16_t* h, int num_pairs, const int32_t* counts,
                           const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                           uint16_t* y, int flags, void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, 1, grid_groups, flags);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!h || !counts || !slot_ids || !group_off || !perm || !y) return SG_ERR_INVALID_ARG;
  return sg::glu_single(arena, h, num_pairs, counts, slot_ids, group_off, perm, grid_groups, y, flags,
                        (cudaStream_t)stream);
}

extern "C" int sg_glu_forward(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                              const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                              const int32_t* perm, int grid_groups, uint16_t* xs, uint16_t* h, uint16_t* y,
                              void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !h || !y) return SG_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const bool permute = sg::use_permute(arena, num_pairs, grid_groups);
  if (permute) {
    if (!xs) return SG_ERR_INVALID_ARG;
    st = sg_permute_rows(x, perm, pair_div, num_pairs, arena->hidden, xs, stream);
    if (st) return st;
  }
  // h in dispatch order, so that the down projection's rows are contiguous
  st = sg::glu_dual(arena, permute ? xs : x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, h,
                    (permute ? SG_IN_DISPATCH_ORDER : 0) | SG_OUT_DISPATCH_ORDER, s);
  if (st) return st;
  return sg::glu_single(arena, h, num_pairs, counts, slot_ids, group_off, perm, grid_groups, y, SG_IN_DISPATCH_ORDER,
                        s);
}

extern "C" int sg_dense_glu(const sg_arena* arena, int sid, const uint16_t* x, int T, uint16_t* h, uint16_t* y,
                            void* stream) {
  int st = sg::check_arena(arena);
  if (st) return st;
  if (T < 0 || sid < 0 || sid >= arena->num_slots) return SG_ERR_INVALID_ARG;
  if (T == 0) return SG_OK;
  if (!x || !h || !y) return SG_ERR_INVALID_ARG;
  if (!sg::tc_supported(arena, true, 1) || !sg::tc_supported(arena, false, 1)) return SG_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  st = sg::tc_dense_launch(arena, true, x, T, sid, h, s);
  if (st) return st;
  return sg::tc_dense_launch(arena, false, h, T, sid, y, s);
}

// ---------------------------------------------------------------- no-alloc variant
// sg_glu_forward with its intermediate rows (h, and the permuted token rows
// when sg_glu_use_permute says so) in a fixed scratch area of this library's
// device memory instead of caller buffers.  The area is a file-scope device
// array, so the call allocates nothing; its address is looked up once per
// device.  No part of it needs to start at zero: every row the down projection
// reads was written by the gate/up launch of the same call.  Calls that overlap
// in time on one device (other streams, other host threads) share the area and
// race; calls on one stream are ordered and safe.
namespace sg {
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64] = {};

static int noalloc_scratch(void** out) {
  int dev = 0;
  SG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    SG_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return SG_OK;
}
}  // namespace sg

extern "C" int sg_glu_forward_noalloc(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                                      const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                                      const int32_t* perm, int grid_groups, uint16_t* y, void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !y) return SG_ERR_INVALID_ARG;
  const size_t h_bytes = ((size_t)num_pairs * arena->inter * 2 + 255) & ~size_t(255);
  const size_t xs_bytes =
      sg::use_permute(arena, num_pairs, grid_groups) ? (size_t)num_pairs * arena->hidden * 2 : 0;
  if (h_bytes + xs_bytes > sg::NOALLOC_SCRATCH_BYTES) return SG_ERR_CAPACITY;
  void* base = nullptr;
  st = sg::noalloc_scratch(&base);
  if (st) return st;
  uint16_t* h = static_cast<uint16_t*>(base);
  uint16_t* xs = xs_bytes ? reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(base) + h_bytes) : nullptr;
  return sg_glu_forward(arena, x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, xs, h, y,
                        stream);
}
