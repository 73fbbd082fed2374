// Gathered SwiGLU expert matmuls over the slot arena (a9, a10, a12):
// streaming GEMV-style kernels for decode steps that touch few experts.
//
// Work item of one warp = (group u, a block of output rows): RW weight rows
// (gate and up rows in pairs for the gate/up projection) x the whole K range.
// A group is one expert slot with the pairs routed to it (sg_dispatch
// layout); the pairs' input rows are staged in shared memory NT at a time.
//
// Bytes in flight decide the speed of a decode GEMV: each lane first issues
// all of its 16-byte weight loads of a K block -- RW rows x NI chunks, 16
// loads, 8 KB per warp -- and the scale/bias words beside them, and only then
// converts and multiplies.  Lane j takes chunks j, j + 32, ... of a row.
// Weights are dequantised in fp32, w = scale * q + bias (q an exact float by
// a magic-number byte permute and one packed subtraction; no bf16 rounding of
// w), and multiplied with the tokens' fp32 values by packed f32x2 FMAs; a
// chunk's x values are read from shared memory once per 8 weights and reused
// across the warp's RW rows.  Partial sums fold across the warp at the end.
#include <mutex>

#include "sg_common.cuh"

namespace sg {

constexpr int GW_WARPS = 4;   // warps (work items) per CTA, all of one group
constexpr int GW_NTMAX = 4;   // pairs staged per pass
constexpr int GW_LOADS = 8;   // 16-byte weight loads per lane per K block (4 KB per warp)

template <int BITS>
struct Wpc {  // weights per 16-byte chunk
  static constexpr int v = BITS == 16 ? 8 : (BITS == 8 ? 16 : 32);
};

__device__ __forceinline__ unsigned long long pk2(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ unsigned long long pk2u(uint32_t lo, uint32_t hi) {
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float lo_f(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

// Weights 8 s .. 8 s + 7 of a 16-byte chunk as four packed fp32 pairs
// (w = scale * q + bias for affine arenas; sb2 = (scale, scale), bb2 =
// (bias, bias)).  q becomes the exact float 2^23 + q by placing its bits in
// the mantissa of 2^23 (0x4B000000), minus 2^23 by one packed add.
template <int BITS>
__device__ __forceinline__ void decode8(const uint4& v, int s, unsigned long long sb2, unsigned long long bb2,
                                        unsigned long long (&w)[4]) {
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
  if (BITS == 16) {  // a bf16 chunk is 8 weights: word q holds weights 2 q, 2 q + 1
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = pk2u(words[q] << 16, words[q] & 0xFFFF0000u);
  } else {
    const unsigned long long m23 = pk2(-8388608.0f, -8388608.0f);
    uint32_t e[8];
    if (BITS == 8) {  // two words = 8 bytes
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t wd = words[2 * s + h];
        // byte m of the word into bits 0-7, zeros above, then the exponent byte of 2^23
        e[4 * h + 0] = __byte_perm(wd, 0x4B000000u, 0x7640);
        e[4 * h + 1] = __byte_perm(wd, 0x4B000000u, 0x7641);
        e[4 * h + 2] = __byte_perm(wd, 0x4B000000u, 0x7642);
        e[4 * h + 3] = __byte_perm(wd, 0x4B000000u, 0x7643);
      }
    } else {  // one word = 8 nibbles, nibble m at bits 4 m
      const uint32_t wd = words[s];
#pragma unroll
      for (int m = 0; m < 8; ++m) e[m] = ((wd >> (4 * m)) & 0xFu) | 0x4B000000u;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = fma2(add2(pk2u(e[2 * q], e[2 * q + 1]), m23), sb2, bb2);
  }
}

// At most 128 registers: four 4-warp CTAs per SM, 16 warps with 4 KB of
// weight loads each in flight.
template <int BITS, bool DUAL, int NI, int NT>
__global__ void __launch_bounds__(GW_WARPS * 32, 4)
gemv_glu_kernel(sg_arena A, const uint16_t* __restrict__ xin, int pair_div, const int32_t* __restrict__ counts,
                const int32_t* __restrict__ slot_ids, const int32_t* __restrict__ group_off,
                const int32_t* __restrict__ perm, uint16_t* __restrict__ out, int in_by_pos, int out_by_pos) {
  constexpr int RW0 = GW_LOADS / NI < 2 ? 2 : (GW_LOADS / NI > 4 ? 4 : GW_LOADS / NI);
  constexpr int RW = RW0 * NT > 16 ? 16 / NT : RW0;  // weight rows per warp (accumulators RW x NT pairs)
  constexpr int ORW = DUAL ? RW / 2 : RW;            // output rows per warp
  constexpr int W = Wpc<BITS>::v;
  constexpr int SUB = BITS == 16 ? 1 : W / 8;        // 8-weight steps per chunk (bf16: one chunk = 8 weights)
  static_assert(!DUAL || RW % 2 == 0, "gate/up rows come in pairs");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // the pairs' rows as fp32, lane-interleaved: the 4 values of (pair b, weight
  // chunk c, 8-weight step, half) sit at float4 slot c % 32 of a 128-float
  // block, so a warp's reads for chunks c0 + lane are contiguous (no bank
  // conflicts) -- [b][c / 32][step][half][c % 32][4]
  float* xs = reinterpret_cast<float*>(smem_raw);
  const int u = blockIdx.y;
  if (u >= counts[0]) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = A.hidden, I = A.inter;
  const int K = DUAL ? H : I;
  const int OUT = DUAL ? I : H;
  const int CPR = K / W;  // 16-byte chunks per row (bf16: K / 8)
  const int NCG = (CPR + 31) / 32;  // 32-chunk groups per row
  auto xs_at = [&](int b, int c, int st, int hf) -> float* {
    return xs + ((((size_t)b * NCG + (c >> 5)) * SUB + st) * 2 + hf) * 128 + (c & 31) * 4;
  };
  const int r0 = (blockIdx.x * GW_WARPS + warp) * ORW;
  const int slot = slot_ids[u];
  const int p_begin = group_off[u], p_end = group_off[u + 1];
  const bool slot_ok = slot >= 0 && slot < A.num_slots;
  const bool rows_ok = r0 < OUT;
  const size_t rbytes = (size_t)K * BITS / 8;
  const int groups = K / 64;

  // matrix m (gate / up, or down) of this slot; row a of the warp is row
  // r0 + a % ORW of matrix a / ORW, clamped so reads stay in range (writes
  // of rows past OUT are masked)
  const size_t slot_row0 = (size_t)(slot_ok ? slot : 0) * OUT;
  const uint8_t* wm[2] = {static_cast<const uint8_t*>(DUAL ? A.gate_w : A.down_w),
                          static_cast<const uint8_t*>(DUAL ? A.up_w : A.down_w)};
  const uint16_t* sm_[2] = {static_cast<const uint16_t*>(DUAL ? A.gate_s : A.down_s),
                            static_cast<const uint16_t*>(DUAL ? A.up_s : A.down_s)};
  const uint16_t* bm[2] = {static_cast<const uint16_t*>(DUAL ? A.gate_b : A.down_b),
                           static_cast<const uint16_t*>(DUAL ? A.up_b : A.down_b)};
  auto row_of = [&](int a) -> size_t { return slot_row0 + min(r0 + (DUAL ? a % ORW : a), OUT - 1); };

  // one K block of this lane's weight chunks and their (scale, bias) words
  auto load_block = [&](int c0, uint4 (&wv)[RW][NI], uint32_t (&sbw)[RW][NI]) {
#pragma unroll
    for (int a = 0; a < RW; ++a) {
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int c = c0 + lane + 32 * i;
        const bool ok = c < CPR;
        const int m = DUAL && a >= ORW;
        const size_t R = row_of(a);
        wv[a][i] = ok ? ldg_nc_v4(wm[m] + R * rbytes + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
        if (BITS != 16) {
          const size_t g = R * groups + c * W / 64;
          sbw[a][i] = ok ? (static_cast<uint32_t>(__ldg(sm_[m] + g)) | (static_cast<uint32_t>(__ldg(bm[m] + g)) << 16))
                         : 0u;
        }
      }
    }
  };

  for (int p0 = p_begin; p0 < p_end; p0 += NT) {
    const int nb = min(NT, p_end - p0);
    uint4 wv[RW][NI];
    uint32_t sbw[RW][NI];
    // the first K block's weights are requested before the pairs' rows are
    // staged, so the two memory round trips overlap
    if (rows_ok && slot_ok) load_block(0, wv, sbw);
    __syncthreads();
    for (int c = threadIdx.x; c < NT * (K / 8); c += blockDim.x) {  // stage the pairs' rows as fp32
      const int b = c / (K / 8), cc = c - b * (K / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (b < nb) {
        const int row = in_by_pos ? p0 + b : perm[p0 + b] / pair_div;
        v = reinterpret_cast<const uint4*>(xin + (size_t)row * K)[cc];
      }
      const int wc = cc * 8 / W, st = (cc * 8 - wc * W) >> 3;  // the weight chunk and 8-weight step of these values
      *reinterpret_cast<float4*>(xs_at(b, wc, st, 0)) = make_float4(lo_bf16(v.x), hi_bf16(v.x), lo_bf16(v.y), hi_bf16(v.y));
      *reinterpret_cast<float4*>(xs_at(b, wc, st, 1)) = make_float4(lo_bf16(v.z), hi_bf16(v.z), lo_bf16(v.w), hi_bf16(v.w));
    }
    __syncthreads();
    if (!rows_ok) continue;
    unsigned long long acc[RW][NT];
#pragma unroll
    for (int a = 0; a < RW; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b) acc[a][b] = 0ull;
    if (slot_ok) {
      for (int c0 = 0; c0 < CPR; c0 += 32 * NI) {
        if (c0 > 0) load_block(c0, wv, sbw);
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          const int c = c0 + lane + 32 * i;
          if (c >= CPR) continue;
#pragma unroll
          for (int sstep = 0; sstep < SUB; ++sstep) {
            // x of these 8 weights for every staged pair, packed in pairs
            unsigned long long x2[NT][4];
#pragma unroll
            for (int b = 0; b < NT; ++b) {
              const float4 lo = *reinterpret_cast<const float4*>(xs_at(b, c, sstep, 0));
              const float4 hi = *reinterpret_cast<const float4*>(xs_at(b, c, sstep, 1));
              x2[b][0] = pk2(lo.x, lo.y);
              x2[b][1] = pk2(lo.z, lo.w);
              x2[b][2] = pk2(hi.x, hi.y);
              x2[b][3] = pk2(hi.z, hi.w);
            }
#pragma unroll
            for (int a = 0; a < RW; ++a) {
              unsigned long long w[4];
              if (BITS == 16) {
                decode8<16>(wv[a][i], 0, 0ull, 0ull, w);
              } else {
                const float s = bf16_to_f32(static_cast<uint16_t>(sbw[a][i] & 0xFFFFu));
                const float bb = bf16_to_f32(static_cast<uint16_t>(sbw[a][i] >> 16));
                decode8<BITS>(wv[a][i], sstep, pk2(s, s), pk2(bb, bb), w);
              }
#pragma unroll
              for (int b = 0; b < NT; ++b)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[a][b] = fma2(w[q], x2[b][q], acc[a][b]);
            }
          }
        }
      }
    }
    // fold: lane (o * NT + b) % 32 writes output row r0 + o of pair b
#pragma unroll
    for (int o = 0; o < ORW; ++o) {
#pragma unroll
      for (int b = 0; b < NT; ++b) {
        if (b >= nb) break;
        const int r = r0 + o;
        const float g = warp_fold_sum(__fadd_rn(lo_f(acc[o][b]), hi_f(acc[o][b])));
        float v2 = 0.0f;
        if (DUAL) v2 = warp_fold_sum(__fadd_rn(lo_f(acc[o + ORW][b]), hi_f(acc[o + ORW][b])));
        if (lane == ((o * NT + b) & 31) && r < OUT) {
          const int p = out_by_pos ? p0 + b : perm[p0 + b];
          uint16_t res = 0;
          if (slot_ok) res = DUAL ? swiglu_bf16(g, v2) : f32_to_bf16(g);
          out[(size_t)p * OUT + r] = res;
        }
      }
    }
  }
}

template <int BITS, bool DUAL, int NI, int NT>
static int launch_gemv_nt(const sg_arena* A, const uint16_t* xin, int pair_div, const int32_t* counts,
                          const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                          uint16_t* out, int in_by_pos, int out_by_pos, cudaStream_t s) {
  constexpr int RW0 = GW_LOADS / NI < 2 ? 2 : (GW_LOADS / NI > 4 ? 4 : GW_LOADS / NI);
  constexpr int RW = RW0 * NT > 16 ? 16 / NT : RW0;
  constexpr int ORW = DUAL ? RW / 2 : RW;
  const int K = DUAL ? A->hidden : A->inter;
  const int OUT = DUAL ? A->inter : A->hidden;
  // lane-interleaved rows: whole 32-chunk groups per row
  const int cpr = K / Wpc<BITS>::v;
  const size_t smem = (size_t)NT * ((cpr + 31) / 32) * 32 * Wpc<BITS>::v * 4;
  if (smem > 48 * 1024) {
    static bool attr_done[64] = {};
    int dev = 0;
    SG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
    if (!attr_done[dev]) {
      SG_CUDA_TRY(cudaFuncSetAttribute(gemv_glu_kernel<BITS, DUAL, NI, NT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
      attr_done[dev] = true;
    }
  }
  const int orows_cta = GW_WARPS * ORW;
  dim3 grid((OUT + orows_cta - 1) / orows_cta, grid_groups);
  gemv_glu_kernel<BITS, DUAL, NI, NT><<<grid, GW_WARPS * 32, smem, s>>>(*A, xin, pair_div, counts, slot_ids,
                                                                        group_off, perm, out, in_by_pos, out_by_pos);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

template <int BITS, bool DUAL, int NI>
static int launch_gemv_ni(const sg_arena* A, int nt, const uint16_t* xin, int pair_div, const int32_t* counts,
                          const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                          uint16_t* out, int in_by_pos, int out_by_pos, cudaStream_t s) {
  if (nt <= 1)
    return launch_gemv_nt<BITS, DUAL, NI, 1>(A, xin, pair_div, counts, slot_ids, group_off, perm, grid_groups, out,
                                             in_by_pos, out_by_pos, s);
  if (nt <= 2)
    return launch_gemv_nt<BITS, DUAL, NI, 2>(A, xin, pair_div, counts, slot_ids, group_off, perm, grid_groups, out,
                                             in_by_pos, out_by_pos, s);
  return launch_gemv_nt<BITS, DUAL, NI, 4>(A, xin, pair_div, counts, slot_ids, group_off, perm, grid_groups, out,
                                           in_by_pos, out_by_pos, s);
}

// NI: chunks per lane per row in one K block, the smallest power of two
// covering the row (at most 4); NT: the staged pairs, from the mean pairs per
// group (a host bound; larger groups take several passes).
template <int BITS, bool DUAL>
static int launch_gemv(const sg_arena* A, const uint16_t* xin, int pair_div, const int32_t* counts,
                       const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                       uint16_t* out, int in_by_pos, int out_by_pos, int num_pairs, cudaStream_t s) {
  const int K = DUAL ? A->hidden : A->inter;
  const int cpr = K / Wpc<BITS>::v;
  const int need = (cpr + 31) / 32;
  const int nt = grid_groups > 0 ? (num_pairs + grid_groups - 1) / grid_groups : 1;
#define SG_GEMV_NI(NIV)                                                                                      \
  return launch_gemv_ni<BITS, DUAL, NIV>(A, nt, xin, pair_div, counts, slot_ids, group_off, perm, grid_groups, \
                                         out, in_by_pos, out_by_pos, s)
  if (need <= 1) SG_GEMV_NI(1);
  if (need <= 2) SG_GEMV_NI(2);
  SG_GEMV_NI(4);  // longer rows take several K blocks
#undef SG_GEMV_NI
}

int check_arena(const sg_arena* A) {
  if (!A || !A->gate_w || !A->up_w || !A->down_w) return SG_ERR_INVALID_ARG;
  if (A->num_slots < 1 || A->hidden < 64 || A->inter < 64) return SG_ERR_SHAPE;
  if (A->hidden % 64 || A->inter % 64) return SG_ERR_SHAPE;
  if ((size_t)A->hidden * 4 * GW_NTMAX > 160 * 1024 || (size_t)A->inter * 4 * GW_NTMAX > 160 * 1024) return SG_ERR_SHAPE;
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
bool i8_supported(const sg_arena* A, bool dual, int grid_groups);
int i8_glu_launch(const sg_arena* A, bool dual, const int8_t* pieces, const float* ex, int in_rows, int pair_div,
                  int in_by_pos, int out_by_pos, const int32_t* counts, const int32_t* slot_ids,
                  const int32_t* group_off, const int32_t* perm, int grid_groups, int num_pairs, uint16_t* out,
                  cudaStream_t s);
int set_i8_tile(int bn);
int quantize_pieces(const uint16_t* x, int rows, int K, int order, int8_t* pieces, float* ex, cudaStream_t s,
                    const int32_t* perm = nullptr, int pair_div = 1, int in_pos = 0,
                    const int32_t* counts = nullptr, const int32_t* group_off = nullptr);
// 0 auto, 1 streaming GEMV, 2 tcgen05 (dequantising), 3 tcgen05 over permuted
// rows, 4 tcgen05 with the integer-operand gate/up wherever it applies
static int g_glu_path = 0;

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

// auto: the tensor-core kernels once the mean pairs per group reaches 4 or
// the groups make at least one weight tile per SM (128 rows for gate/up, 256
// for down); the GEMV serves the smaller steps -- a few experts, a pair or two
// each -- whose tiles would leave most SMs idle (measured: one token through
// 10 experts, the GEMV streams 0.19 of the copy bandwidth, the tensor-core
// kernels 0.13).
static bool use_tc(const sg_arena* A, bool dual, int P, int grid_groups) {
  if (g_glu_path == 1 || !tc_supported(A, dual, grid_groups)) return false;
  if (g_glu_path >= 2) return true;
  const int out = dual ? A->inter : A->hidden;
  const long long tiles = (long long)grid_groups * (out / (dual ? 128 : 256));
  return P >= 4 * grid_groups || tiles >= sm_count();
}

// Whether sg_glu_forward first copies the pairs' token rows into dispatch
// order: worth it once a group's pairs fill 64-wide tiles (a contiguous
// tile of rows then loads with one TMA box per stage).
static bool use_i8(const sg_arena* A, bool dual, int P, int grid_groups);
static bool use_permute(const sg_arena* A, int P, int grid_groups) {
  if (!use_tc(A, true, P, grid_groups) || !use_tc(A, false, P, grid_groups)) return false;
  if (use_i8(A, true, P, grid_groups)) return false;  // the integer-operand gate/up reads the rows in place
  if (g_glu_path == 3) return true;
  return P >= 32 * grid_groups;
}

// The integer-operand kernels (8-bit arenas, gate/up when dual, else down):
// in auto mode wherever the tensor-core path runs with pair tiles of 16
// (decode batches); they need a caller work area for the input rows' pieces.
static bool use_i8(const sg_arena* A, bool dual, int P, int grid_groups) {
  if (g_glu_path == 1 || g_glu_path == 2 || g_glu_path == 3) return false;
  if (grid_groups <= 0 || !i8_supported(A, dual, grid_groups) || !use_tc(A, dual, P, grid_groups)) return false;
  if (g_glu_path == 4) return true;
  return (P + grid_groups - 1) / grid_groups <= 16;
}

// Work area of the pieces of `rows` input rows of the projection's K
// (hidden for gate/up, inter for down): [rows, 2, K] int8, then (256-byte
// aligned) [rows, K / 64, 2] fp32.
static size_t pieces_bytes(const sg_arena* A, bool dual, int rows, size_t* ex_off) {
  const int K = dual ? A->hidden : A->inter;
  const size_t p = ((size_t)rows * 2 * K + 255) & ~size_t(255);
  if (ex_off) *ex_off = p;
  return p + (size_t)rows * (K / 64) * 8;
}

// Rows of pieces the integer-operand kernel reads: the token rows when several
// pairs share one (pair_div > 1: the layer's top-k), else one row per pair
// position in dispatch order (rows per pair: expert-parallel inboxes, h), of
// which only the filled positions are split.
static int piece_rows(bool dual, int in_rows, int num_pairs, int pair_div) {
  return dual && pair_div > 1 ? in_rows : num_pairs;
}

// Input rows' pieces into `work`, then the integer-operand kernel.
static int i8_run(const sg_arena* A, bool dual, const uint16_t* in, int in_rows, int num_pairs, int pair_div,
                  int in_pos, int out_pos, const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                  const int32_t* perm, int grid_groups, uint16_t* out, void* work, size_t work_bytes,
                  cudaStream_t s) {
  const bool by_token = dual && pair_div > 1 && !in_pos;
  const int rows = by_token ? in_rows : num_pairs;
  size_t ex_off = 0;
  if (pieces_bytes(A, dual, rows, &ex_off) > work_bytes) return SG_ERR_CAPACITY;
  int8_t* pieces = static_cast<int8_t*>(work);
  float* ex = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + ex_off);
  // 4-bit weights unpack with nibbles 0,2,4,6 before 1,3,5,7: the pieces follow that order
  const int order = A->bits == 4 ? 1 : 0;
  const int K = dual ? A->hidden : A->inter;
  int st = by_token ? quantize_pieces(in, rows, K, order, pieces, ex, s)
                    : quantize_pieces(in, rows, K, order, pieces, ex, s, perm, pair_div, in_pos, counts, group_off);
  if (st) return st;
  // per-pair pieces are in dispatch order: the kernel reads row pos
  return i8_glu_launch(A, dual, pieces, ex, rows, by_token ? pair_div : 1, by_token ? 0 : 1, out_pos, counts,
                       slot_ids, group_off, perm, grid_groups, num_pairs, out, s);
}

// xs[pos] = x[perm[pos] / pair_div]: one warp per row, 16-byte chunks.  With
// counts / group_off, only the filled positions pos < group_off[counts[0]]
// (ids of -1 leave perm's tail unwritten).
__global__ void __launch_bounds__(256)
permute_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm, int pair_div, int P, int H,
                    uint16_t* __restrict__ xs, const int32_t* __restrict__ counts,
                    const int32_t* __restrict__ group_off) {
  const int pos = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= P) return;
  if (counts && pos >= group_off[counts[0]]) return;
  const int row = perm[pos] / pair_div;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)pos * H);
  for (int c = threadIdx.x & 31; c < H / 8; c += 32) dst[c] = ldg_nc_v4(src + c);
}

static int glu_dual(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div, const int32_t* counts,
                    const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                    uint16_t* h, int flags, cudaStream_t s, void* work = nullptr, size_t work_bytes = 0) {
  const int in_pos = (flags & SG_IN_DISPATCH_ORDER) != 0, out_pos = (flags & SG_OUT_DISPATCH_ORDER) != 0;
  const int div = in_pos ? 1 : pair_div;
  if (work && use_i8(arena, true, num_pairs, grid_groups)) {
    const int in_rows = in_pos ? num_pairs : (num_pairs + pair_div - 1) / pair_div;
    return i8_run(arena, true, x, in_rows, num_pairs, div, in_pos, out_pos, counts, slot_ids, group_off, perm,
                  grid_groups, h, work, work_bytes, s);
  }
  if (use_tc(arena, true, num_pairs, grid_groups)) {
    const int in_rows = in_pos ? num_pairs : (num_pairs + pair_div - 1) / pair_div;
    return tc_glu_launch(arena, true, x, in_rows, div, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, h, s);
  }
  switch (arena->bits) {
    case 16: return launch_gemv<16, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, num_pairs, s);
    case 8: return launch_gemv<8, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, num_pairs, s);
    default: return launch_gemv<4, true>(arena, x, div, counts, slot_ids, group_off, perm, grid_groups, h, in_pos, out_pos, num_pairs, s);
  }
}

static int glu_single(const sg_arena* arena, const uint16_t* h, int num_pairs, const int32_t* counts,
                      const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm, int grid_groups,
                      uint16_t* y, int flags, cudaStream_t s, void* work = nullptr, size_t work_bytes = 0) {
  const int in_pos = (flags & SG_IN_DISPATCH_ORDER) != 0, out_pos = (flags & SG_OUT_DISPATCH_ORDER) != 0;
  if (work && use_i8(arena, false, num_pairs, grid_groups))
    return i8_run(arena, false, h, num_pairs, num_pairs, 1, in_pos, out_pos, counts, slot_ids, group_off, perm,
                  grid_groups, y, work, work_bytes, s);
  if (use_tc(arena, false, num_pairs, grid_groups))
    return tc_glu_launch(arena, false, h, num_pairs, 1, in_pos, out_pos, num_pairs, counts, slot_ids, group_off, perm,
                         grid_groups, y, s);
  switch (arena->bits) {
    case 16: return launch_gemv<16, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, num_pairs, s);
    case 8: return launch_gemv<8, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, num_pairs, s);
    default: return launch_gemv<4, false>(arena, h, 1, counts, slot_ids, group_off, perm, grid_groups, y, in_pos, out_pos, num_pairs, s);
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

extern "C" int sg_set_glu_tile(int bn) { return sg::set_i8_tile(bn); }

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
  sg::permute_rows_kernel<<<(num_pairs + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, perm, pair_div, num_pairs, H, xs,
                                                                                  nullptr, nullptr);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_permute_pairs(const uint16_t* x, const int32_t* perm, int pair_div, const int32_t* counts,
                                const int32_t* group_off, int num_pairs, int H, uint16_t* xs, void* stream) {
  if (num_pairs < 0 || pair_div < 1) return SG_ERR_INVALID_ARG;
  if (H < 8 || H % 8) return SG_ERR_SHAPE;
  if (num_pairs == 0) return SG_OK;
  if (!x || !perm || !counts || !group_off || !xs) return SG_ERR_INVALID_ARG;
  sg::permute_rows_kernel<<<(num_pairs + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, perm, pair_div, num_pairs, H, xs,
                                                                                  counts, group_off);
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

namespace sg {
// Scratch of sg_glu_forward: the permuted token rows (prefill-sized groups),
// or the pieces of the token rows for the integer-operand gate/up and then,
// in the same bytes, the pieces of h for the integer-operand down projection.
static size_t forward_scratch(const sg_arena* A, int P, int pair_div, int gg, size_t* gu, size_t* dn) {
  *gu = use_i8(A, true, P, gg) ? pieces_bytes(A, true, piece_rows(true, (P + pair_div - 1) / pair_div, P, pair_div),
                                              nullptr)
                                 : 0;
  *dn = use_i8(A, false, P, gg) ? pieces_bytes(A, false, P, nullptr) : 0;
  if (use_permute(A, P, gg)) return (size_t)P * A->hidden * 2;
  return *gu > *dn ? *gu : *dn;
}
}  // namespace sg

extern "C" int sg_glu_forward(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                              const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                              const int32_t* perm, int grid_groups, void* scratch, uint16_t* h, uint16_t* y,
                              void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !h || !y) return SG_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const bool permute = sg::use_permute(arena, num_pairs, grid_groups);
  uint16_t* xs = static_cast<uint16_t*>(scratch);
  if (permute) {
    if (!xs) return SG_ERR_INVALID_ARG;
    // the filled positions only (the dispatch leaves perm's tail unwritten when ids hold -1)
    sg::permute_rows_kernel<<<(num_pairs + 7) / 8, 256, 0, s>>>(x, perm, pair_div, num_pairs, arena->hidden, xs,
                                                                 counts, group_off);
    SG_LAUNCH_CHECK();
  }
  // h in dispatch order, so that the down projection's rows are contiguous.
  // Without scratch the integer-operand kernels are not used.
  size_t gu = 0, dn = 0;
  sg::forward_scratch(arena, num_pairs, pair_div, grid_groups, &gu, &dn);
  void* work = permute ? nullptr : scratch;
  st = sg::glu_dual(arena, permute ? xs : x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, h,
                    (permute ? SG_IN_DISPATCH_ORDER : 0) | SG_OUT_DISPATCH_ORDER, s, work, work ? gu : 0);
  if (st) return st;
  return sg::glu_single(arena, h, num_pairs, counts, slot_ids, group_off, perm, grid_groups, y, SG_IN_DISPATCH_ORDER,
                        s, work, work ? dn : 0);
}

extern "C" long long sg_glu_forward_scratch_bytes(const sg_arena* arena, int num_pairs, int pair_div,
                                                  int grid_groups) {
  const int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0) return 0;
  size_t gu = 0, dn = 0;
  return (long long)sg::forward_scratch(arena, num_pairs, pair_div, grid_groups, &gu, &dn);
}

extern "C" long long sg_glu_gate_up_work_bytes(const sg_arena* arena, int num_pairs, int pair_div, int grid_groups,
                                               int flags) {
  const int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, flags);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0 || !sg::use_i8(arena, true, num_pairs, grid_groups)) return 0;
  const bool in_pos = (flags & SG_IN_DISPATCH_ORDER) != 0;
  const int rows = in_pos ? num_pairs : sg::piece_rows(true, (num_pairs + pair_div - 1) / pair_div, num_pairs, pair_div);
  return (long long)sg::pieces_bytes(arena, true, rows, nullptr);
}

extern "C" int sg_glu_gate_up_work(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                                   const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                                   const int32_t* perm, int grid_groups, uint16_t* h, int flags, void* work,
                                   long long work_bytes, void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, pair_div, grid_groups, flags);
  if (st) return st;
  if (work_bytes < 0) return SG_ERR_INVALID_ARG;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!x || !counts || !slot_ids || !group_off || !perm || !h) return SG_ERR_INVALID_ARG;
  return sg::glu_dual(arena, x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, h, flags,
                      (cudaStream_t)stream, work_bytes > 0 ? work : nullptr, static_cast<size_t>(work_bytes));
}

extern "C" long long sg_glu_down_work_bytes(const sg_arena* arena, int num_pairs, int grid_groups) {
  const int st = sg::check_glu_args(arena, num_pairs, 1, grid_groups, 0);
  if (st) return st;
  if (num_pairs == 0 || grid_groups == 0 || !sg::use_i8(arena, false, num_pairs, grid_groups)) return 0;
  return (long long)sg::pieces_bytes(arena, false, num_pairs, nullptr);
}

extern "C" int sg_glu_down_work(const sg_arena* arena, const uint16_t* h, int num_pairs, const int32_t* counts,
                                const int32_t* slot_ids, const int32_t* group_off, const int32_t* perm,
                                int grid_groups, uint16_t* y, int flags, void* work, long long work_bytes,
                                void* stream) {
  int st = sg::check_glu_args(arena, num_pairs, 1, grid_groups, flags);
  if (st) return st;
  if (work_bytes < 0) return SG_ERR_INVALID_ARG;
  if (num_pairs == 0 || grid_groups == 0) return SG_OK;
  if (!h || !counts || !slot_ids || !group_off || !perm || !y) return SG_ERR_INVALID_ARG;
  return sg::glu_single(arena, h, num_pairs, counts, slot_ids, group_off, perm, grid_groups, y, flags,
                        (cudaStream_t)stream, work_bytes > 0 ? work : nullptr, static_cast<size_t>(work_bytes));
}

extern "C" int sg_quantize_pieces(const uint16_t* x, int rows, int K, int order, int8_t* pieces, float* ex,
                                  void* stream) {
  if (rows < 0 || (order != 0 && order != 1)) return SG_ERR_INVALID_ARG;
  if (K < 64 || K % 64) return SG_ERR_SHAPE;
  if (rows == 0) return SG_OK;
  if (!x || !pieces || !ex) return SG_ERR_INVALID_ARG;
  return sg::quantize_pieces(x, rows, K, order, pieces, ex, (cudaStream_t)stream);
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
  // the permuted token rows or the token rows' pieces, as sg_glu_forward uses them
  const long long xs_need = sg_glu_forward_scratch_bytes(arena, num_pairs, pair_div, grid_groups);
  if (xs_need < 0) return static_cast<int>(xs_need);
  const size_t xs_bytes = static_cast<size_t>(xs_need);
  if (h_bytes + xs_bytes > sg::NOALLOC_SCRATCH_BYTES) return SG_ERR_CAPACITY;
  void* base = nullptr;
  st = sg::noalloc_scratch(&base);
  if (st) return st;
  uint16_t* h = static_cast<uint16_t*>(base);
  void* xs = xs_bytes ? static_cast<void*>(static_cast<uint8_t*>(base) + h_bytes) : nullptr;
  return sg_glu_forward(arena, x, num_pairs, pair_div, counts, slot_ids, group_off, perm, grid_groups, xs, h, y,
                        stream);
}
