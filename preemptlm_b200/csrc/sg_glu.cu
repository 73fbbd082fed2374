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
#include <cuda_fp16.h>

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
                  const int32_t* perm, int grid_groups, uint16_t* out, const float* xsum, const float* xscale,
                  cudaStream_t s);
bool tc_fq_supported(const sg_arena* A, int P, int grid_groups);
int tc_dense_launch(const sg_arena* A, bool dual, const uint16_t* in, int rows, int sid, uint16_t* out,
                    cudaStream_t s);
// 0 auto, 1 streaming GEMV, 2 tcgen05, 3 tcgen05 over permuted rows, 4 tcgen05
// with the exact dequantised weights (no factored scales)
static int g_glu_path = 0;

// auto: the tensor-core path once the mean pairs per group reaches 2
static bool use_tc(const sg_arena* A, bool dual, int P, int grid_groups) {
  if (g_glu_path == 1 || !tc_supported(A, dual, grid_groups)) return false;
  if (g_glu_path >= 2) return true;
  return P >= 2 * grid_groups;
}

// Whether sg_glu_forward first copies the pairs' token rows into dispatch
// order: worth it once a group's pairs fill 64-wide tiles (a contiguous
// tile of rows then loads with one TMA box per stage).
static bool use_permute(const sg_arena* A, int P, int grid_groups) {
  if (!use_tc(A, true, P, grid_groups) || !use_tc(A, false, P, grid_groups)) return false;
  if (g_glu_path == 3) return true;
  return P >= 32 * grid_groups;
}

// Whether sg_glu_forward's gate/up takes factored scales over prepared f16
// rows (decode-sized groups of a quantised arena).
static bool use_fq(const sg_arena* A, int P, int grid_groups) {
  return g_glu_path != 4 && use_tc(A, true, P, grid_groups) && tc_fq_supported(A, P, grid_groups);
}

// Prepared-row scratch of sg_glu_prep: R rows of x16 [R][K] f16, then
// xsum [R][K/64] fp32, then xscale [R] fp32, each part 256-byte aligned.
static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
struct PrepLayout {
  size_t x16, xsum, xscale, bytes;
};
static PrepLayout prep_layout(int R, int K) {
  PrepLayout l;
  l.x16 = 0;
  l.xsum = align256((size_t)R * K * 2);
  l.xscale = l.xsum + align256((size_t)R * (K / 64) * 4);
  l.bytes = l.xscale + align256((size_t)R * 4);
  return l;
}

// FQ row preparation, one warp per prepared row i (source row perm[i] /
// pair_div when permuted, else i): e = the power of two that brings the row's
// largest magnitude into [2^14, 2^15); x16 = f16(x * 2^-e), exact for every
// value within 2^28 of that maximum; xsum[i][g] = fp32 sum of the 64 f16
// values of group g (8 in a lane, then 8 lanes); xscale[i] = 2^e.  Rows
// without a source (a permutation entry out of range) are zero.
__global__ void __launch_bounds__(256)
fq_prep_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm, int pair_div, int permuted, int R,
               int src_rows, int K, uint16_t* __restrict__ x16, float* __restrict__ xsum,
               float* __restrict__ xscale) {
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= R) return;
  const int src = permuted ? perm[i] / pair_div : i;
  const bool valid = src >= 0 && src < src_rows;
  const uint16_t* row = x + (size_t)(valid ? src : 0) * K;
  const int chunks = K >> 3, G = K >> 6;
  uint32_t m = 0;  // largest |x| as bf16 magnitude bits
  for (int c = lane; c < chunks && valid; c += 32) {
    const uint4 v = ldg_nc_v4(row + (size_t)c * 8);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) m = max(m, max(w[q] & 0x7FFFu, (w[q] >> 16) & 0x7FFFu));
  }
  m = __reduce_max_sync(0xffffffffu, m);
  const int ebits = static_cast<int>(m >> 7);  // bf16 exponent field (fp32's)
  const int e = ebits == 0 ? 0 : max(ebits - 141, -126);
  const float down = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
  uint4* orow = reinterpret_cast<uint4*>(x16 + (size_t)i * K);
  for (int base = 0; base < chunks; base += 32) {
    const int c = base + lane;
    const bool act = c < chunks;  // uniform across each 8-lane group (chunks % 8 == 0)
    float sum = 0.f;
    if (act) {
      const uint4 v = valid ? ldg_nc_v4(row + (size_t)c * 8) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 h = __floats2half2_rn(__fmul_rn(__uint_as_float(w[q] << 16), down),
                                            __fmul_rn(__uint_as_float(w[q] & 0xFFFF0000u), down));
        const float2 f = __half22float2(h);
        sum = __fadd_rn(__fadd_rn(sum, f.x), f.y);
        o[q] = *reinterpret_cast<const uint32_t*>(&h);
      }
      orow[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 4));
    if (act && (lane & 7) == 0) xsum[(size_t)i * G + (c >> 3)] = sum;
  }
  if (lane == 0) xscale[i] = valid ? __uint_as_float(static_cast<uint32_t>(127 + e) << 23) : 0.f;
}

// Rows of the prepared scratch: every pair in dispatch order when permuted,
// else the token rows.
static int prep_rows(const sg_arena* A, int P, int pair_div, int grid_groups) {
  return use_permute(A, P, grid_groups) ? P : (P + pair_div - 1) / pair_div;
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
  const int in_rows = in_pos ? num_pairs : (num_pairs + pair_div - 1) / pair_div;
  if (flags & SG_IN_PREPARED) {
    // x is sg_glu_prep's scratch: f16 rows, group sums, row scales
    if (!use_fq(arena, num_pairs, grid_groups)) return SG_ERR_SHAPE;
    const PrepLayout l = prep_layout(in_rows, arena->hidden);
    const uint8_t* base = reinterpret_cast<const uint8_t*>(x);
    return tc_glu_launch(arena, true, x, in_rows, div, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, h, reinterpret_cast<const float*>(base + l.xsum),
                         reinterpret_cast<const float*>(base + l.xscale), s);
  }
  if (use_tc(arena, true, num_pairs, grid_groups)) {
    return tc_glu_launch(arena, true, x, in_rows, div, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, h, nullptr, nullptr, s);
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
                         grid_groups, y, nullptr, nullptr, s);
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
  if (flags & ~(SG_IN_DISPATCH_ORDER | SG_OUT_DISPATCH_ORDER | SG_IN_PREPARED)) return SG_ERR_INVALID_ARG;
  if (grid_groups > 65535) return SG_ERR_SHAPE;
  return SG_OK;
}
}  // namespace sg

extern "C" int sg_set_glu_path(int mode) {
  if (mode < 0 || mode > 4) return SG_ERR_INVALID_ARG;
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

extern "C" long long sg_glu_scratch_bytes(const sg_arena* arena, int num_pairs, int pair_div, int grid_groups) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return 0;
  if (sg::use_fq(arena, num_pairs, grid_groups))
    return (long long)sg::prep_layout(sg::prep_rows(arena, num_pairs, pair_div, grid_groups), arena->hidden).bytes;
  if (sg::use_permute(arena, num_pairs, grid_groups)) return (long long)num_pairs * arena->hidden * 2;
  return 0;
}

extern "C" int sg_glu_prep(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                           const int32_t* perm, int grid_groups, void* scratch, void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return 0;
  if (!x || !perm) return SG_ERR_INVALID_ARG;
  const bool permute = sg::use_permute(arena, num_pairs, grid_groups);
  if (sg::use_fq(arena, num_pairs, grid_groups)) {
    if (!scratch) return SG_ERR_INVALID_ARG;
    const int R = sg::prep_rows(arena, num_pairs, pair_div, grid_groups);
    const int src_rows = (num_pairs + pair_div - 1) / pair_div;
    const sg::PrepLayout l = sg::prep_layout(R, arena->hidden);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    sg::fq_prep_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
        x, perm, pair_div, permute ? 1 : 0, R, src_rows, arena->hidden, reinterpret_cast<uint16_t*>(base + l.x16),
        reinterpret_cast<float*>(base + l.xsum), reinterpret_cast<float*>(base + l.xscale));
    SG_LAUNCH_CHECK();
    return SG_IN_PREPARED | (permute ? SG_IN_DISPATCH_ORDER : 0);
  }
  if (permute) {
    if (!scratch) return SG_ERR_INVALID_ARG;
    st = sg_permute_rows(x, perm, pair_div, num_pairs, arena->hidden, static_cast<uint16_t*>(scratch), stream);
    return st ? st : SG_IN_DISPATCH_ORDER;
  }
  return 0;
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
  if (flags & SG_IN_PREPARED) return SG_ERR_INVALID_ARG;  // gate/up input only
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!h || !counts || !slot_ids || !group_off || !perm || !y) return SG_ERR_INVALID_ARG;
  return sg::glu_single(arena, h, num_pairs, counts, slot_ids, group_off, perm, grid_groups, y, flags,
                        (cudaStream_t)stream);
}

extern "C" int sg_glu_forward(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                              const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                              const int32_t* perm, int grid_groups, void* xs, uint16_t* h, uint16_t* y,
                              void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !h || !y) return SG_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int in_flags = sg_glu_prep(arena, x, num_pairs, pair_div, perm, grid_groups, xs, stream);
  if (in_flags < 0) return in_flags;
  // h in dispatch order, so that the down projection's rows are contiguous
  st = sg::glu_dual(arena, in_flags ? static_cast<const uint16_t*>(xs) : x, num_pairs, pair_div, counts, slot_ids,
                    group_off, perm, grid_groups, h, in_flags | SG_OUT_DISPATCH_ORDER, s);
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
// sg_glu_forward with its intermediate rows (h, and the prepared token rows
// when sg_glu_scratch_bytes asks for them) in a fixed scratch area of this library's
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
  const long long xs_need = sg_glu_scratch_bytes(arena, num_pairs, pair_div, grid_groups);
  if (xs_need < 0) return (int)xs_need;
  const size_t xs_bytes = (size_t)xs_need;
  if (h_bytes + xs_bytes > sg::NOALLOC_SCRATCH_BYTES) return SG_ERR_CAPACITY;
  void* base = nullptr;
  st = sg::noalloc_scratch(&base);
  if (st) return st;
  uint16_t* h = static_cast<uint16_t*>(base);
  void* xs = xs_bytes ? static_cast<void*>(static_cast<uint8_t*>(base) + h_bytes) : nullptr;
  return sg_glu_forward(arena, x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, xs, h, y,
                        stream);
}
