// Integer-operand gathered gate/up for quantised arenas at decode tile widths
// (a9, a10, a12).  Included by sg_glu_tc.cu: it shares that translation
// unit's PTX helpers and device status word.
//
// The affine weights are never dequantised.  With w[m,k] = s[m,g] q[m,k] +
// b[m,g] (g = k / 64),
//
//   sum_k w[m,k] x[n,k] = sum_g s[m,g] * (sum_{k in g} q[m,k] x[n,k])
//                       + sum_g b[m,g] * (sum_{k in g} x[n,k]).
//
// The token rows are first split into 8-bit pieces per 64-group
// (sg_quantize_pieces): x[n,k] = E[n,g] * (256 hi[n,k] + lo[n,k]), E a power
// of two chosen so the group's largest |x| maps below 2^14 -- every element
// within 2^6 of the group maximum is represented exactly, smaller ones to
// 2^-14 of the maximum.  The tensor cores then multiply the raw unsigned
// 8-bit weights (the arena's q8 rows, loaded by TMA straight into the MMA
// operand layout) with the signed pieces (tcgen05.mma kind::i8, exact int32
// accumulation), one TMEM accumulator per 64-group: D[m, j] = sum q hi and
// D[m, BN + j] = sum q lo for the tile's BN pairs j.  The epilogue warps fold
// each group: y[m,j] += s[m,g] * (E[j,g] * float(256 D_hi + D_lo)) +
// b[m,g] * X[j,g], X = E * sum(256 hi + lo), and finish with SwiGLU.
//
// Warp roles (11 warps, one CTA per SM, persistent over the tile list of the
// dequantising kernel):
//   w0      TMA producer: 128 rows x 128 bytes of gate and of up per stage
//           (K = 128), and the tiles' scale/bias chunks (8 groups x 128 rows)
//   w1      TMEM allocation + single-thread tcgen05.mma issue: two K = 32
//           MMAs per matrix per group into a ring of 8 group accumulators
//   w2      B producer: the pairs' hi/lo piece rows by 16-byte cp.async into
//           the SW128 operand layout; per tile, the pairs' (E, X) table
//   w3-w10  epilogue: warp (quadrant, matrix) folds its 32 rows of one matrix,
//           the up warps hand their sums to the gate warps through shared
//           memory, the gate warps write h = swiglu(gate, up) in bf16
//
// Every wait is bounded as in the dequantising kernel; on expiry the CTA
// records SG_ERR_TIMEOUT, drains its copies, frees TMEM and returns.
#pragma once

namespace sg {
namespace i8 {

using namespace tc;

constexpr int KS = 128;         // K per pipeline stage: one 128-byte swizzle atom of 8-bit operands
constexpr int GSZ = 64;         // quantisation group
constexpr int TILE8_MAX = 6;    // 8-pair tiles while groups average at most this many pairs
constexpr int PIECE_BITS = 14;  // the group maximum maps below 2^PIECE_BITS

// ------------------------------------------------------------------ pieces
// Element value of a bf16 as a signed integer scaled so that biased exponent
// eM (the group maximum's) maps the leading bit to 2^(PIECE_BITS - 1):
//   |v| = m8 * 2^(ex - eM + PIECE_BITS - 8), m8 the 8-bit significand,
// rounded to nearest (ties away from zero) when the shift is negative.
__device__ __forceinline__ int piece_value(uint32_t b16, int eM) {
  const int ex = (b16 >> 7) & 0xFF;
  int m = b16 & 0x7F;
  int e = ex;
  if (ex == 0) {
    e = 1;  // subnormal: no implicit bit
  } else {
    m |= 0x80;
  }
  const int sh = e - eM + (PIECE_BITS - 8);
  int v;
  if (sh >= 0) v = m << sh;
  else if (sh > -31) v = (m + (1 << (-sh - 1))) >> (-sh);
  else v = 0;
  return (b16 & 0x8000u) ? -v : v;
}

// One thread per 8 elements, 8 threads per 64-group.  ORDER 0: pieces in k
// order; ORDER 1 (4-bit arenas): within every 8 elements the order
// 0, 2, 4, 6, 1, 3, 5, 7, the order of the unpacked nibbles.
// Dispatch mode (perm != nullptr): output row pos < rows holds the pieces of
// input row perm[pos] / pair_div (or pos when in_pos), for the pair positions
// pos < group_off[counts[0]] only -- expert-parallel inboxes are padded, and
// their unused entries are never read.
__global__ void __launch_bounds__(256)
quantize_pieces_kernel(const uint16_t* __restrict__ x, int rows, int K, int order, int8_t* __restrict__ pieces,
                       float* __restrict__ ex, const int32_t* __restrict__ perm, int pair_div, int in_pos,
                       const int32_t* __restrict__ counts, const int32_t* __restrict__ group_off) {
  const int G = K / GSZ;
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // chunk of 8 elements
  const long long nchunks = (long long)rows * (K / 8);
  bool live = t < nchunks;
  const long long ci = live ? t : 0;
  const int row = static_cast<int>(ci / (K / 8));
  const int c = static_cast<int>(ci - (long long)row * (K / 8));  // chunk within the row
  int src = row;
  if (perm) {  // the 8 threads of a group share the row, so they agree on `live`
    live = live && row < group_off[counts[0]];
    src = live ? (in_pos ? row : perm[row] / pair_div) : 0;
  }
  const uint4 v = live ? ldg_nc_v4(x + (size_t)src * K + (size_t)c * 8) : make_uint4(0, 0, 0, 0);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t b[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    b[2 * i] = w[i] & 0xFFFFu;
    b[2 * i + 1] = w[i] >> 16;
  }
  // largest biased exponent among the group's nonzero elements (the maximum
  // magnitude's exponent); the 8 threads of a group are 8 consecutive lanes
  int eM = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = (b[i] >> 7) & 0xFF;
    eM = max(eM, (b[i] & 0x7FFFu) ? max(e, 1) : 0);
  }
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) eM = max(eM, __shfl_xor_sync(0xffffffffu, eM, off));
  int iv[8];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    iv[i] = piece_value(b[i], eM);
    sum += iv[i];
  }
  uint32_t hi[2] = {0, 0}, lo[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int src = order ? ((i & 3) * 2 + (i >> 2)) : i;  // element placed at position i
    const int h = (iv[src] + 128) >> 8;                    // arithmetic shift: floor
    const int l = iv[src] - 256 * h;                       // [-128, 127]
    hi[i >> 2] |= (static_cast<uint32_t>(h) & 0xFFu) << (8 * (i & 3));
    lo[i >> 2] |= (static_cast<uint32_t>(l) & 0xFFu) << (8 * (i & 3));
  }
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (!live) return;
  int8_t* prow = pieces + (size_t)row * 2 * K;
  *reinterpret_cast<uint2*>(prow + (size_t)c * 8) = make_uint2(hi[0], hi[1]);
  *reinterpret_cast<uint2*>(prow + K + (size_t)c * 8) = make_uint2(lo[0], lo[1]);
  if ((c & 7) == 0) {
    // E = 2^(eM - 127 - (PIECE_BITS - 1)): a normal or subnormal power of two
    const int e2 = eM - 127 - (PIECE_BITS - 1);
    const float E = e2 >= -126 ? __uint_as_float(static_cast<uint32_t>(e2 + 127) << 23)
                               : __uint_as_float(1u << (e2 + 149));
    float* o = ex + ((size_t)row * G + c / 8) * 2;
    o[0] = E;
    o[1] = static_cast<float>(sum) * E;
  }
}

// ------------------------------------------------------------------ kernel configuration
// BITS 8: the packed rows are the MMA's A operand as they are (TMA into shared
// memory, SA stages).  BITS 4: TMA brings 128 packed bytes (256 weights) of
// every row per stage (SP stages); 8 unpacking warps turn each half into 128
// unsigned bytes per row -- in the order 0,2,4,6,1,3,5,7 within every 8
// weights, the pieces' order 1 -- and store them into tensor memory (SAT
// stages), where the MMAs read A.
template <int BITS, int BN>
struct Cfg {
  static constexpr bool Q4 = BITS == 4;
  static constexpr int NB = 2 * BN;                  // B rows: the pairs' hi pieces, then their lo pieces
  static constexpr int A_MAT = BM * KS;              // one matrix's packed stage: 128 rows x 128 bytes (16 KB)
  static constexpr int A_BYTES = 2 * A_MAT;          // both matrices
  static constexpr int B_BYTES = NB * KS;            // 2 BN rows x 128 bytes
  static constexpr int SA = Q4 ? 0 : 4;              // shared-memory A stages (8-bit)
  static constexpr int SP = Q4 ? 3 : 0;              // packed stages (4-bit), two K stages each
  static constexpr int SAT = Q4 ? 4 : 0;             // tensor-memory A stages (4-bit, unpacked)
  static constexpr int A_TCOLS = 2 * KS / 4;         // TMEM columns of one unpacked stage: 2 matrices x 32
  static constexpr int SB = 6;
  static constexpr int SS = 3;
  static constexpr int S_BYTES = 2 * 2 * BM * 16;    // [matrix][scales, biases][128 rows][8 groups] bf16
  static constexpr int GMAX = 64;                    // groups per row (K <= 4096)
  static constexpr int T_BYTES = GMAX * 2 * BN * 4;  // pair table: [group][E, X][BN] fp32
  static constexpr int X_STRIDE = BN + 4;            // hand-off rows: BN fp32 + padding
  static constexpr int X_BYTES = BM * X_STRIDE * 4;
  static constexpr int ACC_COLS = 2 * NB;            // one group: gate and up, NB columns each
  // group accumulators in flight: what tensor memory leaves after the A stages
  static constexpr int RINGN = cmin(16, (512 - SAT * A_TCOLS) / ACC_COLS);
  static constexpr int ACC_TOTAL = RINGN * ACC_COLS;
  static constexpr int TMEM_COLS = ACC_TOTAL + SAT * A_TCOLS;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + (SA + SP) * A_BYTES;
  static constexpr int OFF_S = OFF_B + SB * B_BYTES;
  static constexpr int OFF_T = OFF_S + SS * S_BYTES;
  static constexpr int OFF_X = OFF_T + 2 * T_BYTES;
  static constexpr int OFF_PLAN = OFF_X + 2 * X_BYTES;
  static constexpr int OFF_BAR = (OFF_PLAN + (PLAN_MAX_GROUPS + 1) * 4 + 15) & ~15;
  static constexpr int NUM_BARS = 2 * (SA + SAT) + 2 * SP + 2 * SB + 2 * RINGN + 2 * SS + 2 * 2 + 2 * 2;
  static constexpr int SMEM = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
  static constexpr int EPI_WARP0 = 3;
  static constexpr int UNP_WARP0 = EPI_WARP0 + 8;    // 4-bit: the unpacking warps follow the epilogue
  static constexpr int THREADS = (UNP_WARP0 + (Q4 ? 8 : 0)) * 32;
  static_assert(TMEM_COLS == 512, "tensor memory budget");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(B_BYTES % 1024 == 0, "B stages keep 1024-byte alignment");
};

// Instruction descriptor, kind::i8: D s32, A unsigned 8-bit (the raw weights),
// B signed 8-bit (the pieces), both K-major, M = 128, N = NB.
template <int NB>
__device__ __forceinline__ uint32_t idesc_i8() {
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(NB >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// A from tensor memory: row m in lane m, four consecutive K bytes per column
__device__ __forceinline__ void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// NB columns of the warp's 32 lanes: the hi sums of the tile's pairs, then the lo sums
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld32(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }

struct Args {
  int num_slots, K, OUT;
  const int8_t* pieces;  // [in_rows, 2, K]: hi then lo pieces of every input row
  const float* ex;       // [in_rows, K / 64, 2]: (E, X) per group
  int in_rows;
  const int32_t* counts;
  const int32_t* slot_ids;
  const int32_t* group_off;
  const int32_t* perm;
  int pair_div;    // input row of pair position pos: perm[pos] / pair_div, or pos when in_by_pos
  int in_by_pos;
  int out_by_pos;  // output row: pos, or perm[pos]
  int max_groups;
  uint16_t* out;
};

// Tile t of the flat list: weight-row tile m, group u (the largest u with
// plan[u] <= n-tile index), its first pair n0 and valid pair count.
struct ITile {
  int u, m, n0, nvalid, slot, goff;
};
template <int BN>
__device__ __forceinline__ ITile itile_of(int t, const int* plan, int U, int NT, const Args& a) {
  ITile tl;
  tl.m = t / NT;
  const int fn = t - tl.m * NT;
  int lo = 0, hi = U;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (plan[mid] <= fn) lo = mid;
    else hi = mid;
  }
  tl.u = lo;
  tl.n0 = (fn - plan[lo]) * BN;
  tl.goff = a.group_off[lo];
  tl.nvalid = min(BN, a.group_off[lo + 1] - tl.goff - tl.n0);
  tl.slot = a.slot_ids[lo];
  return tl;
}

// ------------------------------------------------------------------ the kernel
// MODE 1: gate/up, the two matrices of a 128-row tile and the SwiGLU
// hand-off; MODE 2: down projection, the two 128-row halves of a 256-row
// tile (the same bytes per stage), written straight out.
template <int BITS, int MODE, int BN>
__global__ void __launch_bounds__(Cfg<BITS, BN>::THREADS, 1)
glu_i8_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
              const __grid_constant__ CUtensorMap tmS0, const __grid_constant__ CUtensorMap tmQ0,
              const __grid_constant__ CUtensorMap tmS1, const __grid_constant__ CUtensorMap tmQ1, const Args args) {
  using C = Cfg<BITS, BN>;
  constexpr int NB = C::NB;
  constexpr int NA = C::SA + C::SAT;  // A stages (shared or tensor memory)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sS = smem + C::OFF_S;
  float* sT = reinterpret_cast<float*>(smem + C::OFF_T);
  float* sX = reinterpret_cast<float*>(smem + C::OFF_X);
  int* plan = reinterpret_cast<int*>(smem + C::OFF_PLAN);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  // A stage ready: TMA tx (8-bit) or the 8 unpacking warps (4-bit); consumed: MMA commit
  uint64_t* a_full = bars;                   // [NA]
  uint64_t* a_empty = a_full + NA;           // [NA]
  uint64_t* p_full = a_empty + NA;           // [SP] packed stage landed (TMA tx, 4-bit)
  uint64_t* p_empty = p_full + C::SP;        // [SP] packed stage read (8 unpacking warps)
  uint64_t* b_full = p_empty + C::SP;        // [SB] piece rows landed (32 cp.async arrivals)
  uint64_t* b_empty = b_full + C::SB;        // [SB] piece rows consumed (MMA commit)
  uint64_t* acc_full = b_empty + C::SB;      // [RINGN] group accumulator ready (MMA commit)
  uint64_t* acc_empty = acc_full + C::RINGN;  // [RINGN] group accumulator read (8 epilogue warps)
  uint64_t* s_full = acc_empty + C::RINGN;   // [SS] scale/bias chunk landed (TMA tx)
  uint64_t* s_empty = s_full + C::SS;        // [SS] scale/bias chunk read (8 epilogue warps)
  uint64_t* t_full = s_empty + C::SS;        // [2] pair table written (32 producer lanes)
  uint64_t* t_empty = t_full + 2;            // [2] pair table read (8 epilogue warps)
  uint64_t* x_full = t_empty + 2;            // [2] up sums handed over (128 up threads)
  uint64_t* x_empty = x_full + 2;            // [2] up sums taken (128 gate threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Ctl ctl{abort_flag};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = args.K;
  const int NKS = K / KS;
  const int G = K / GSZ;
  constexpr int TR = MODE == 2 ? 2 * BM : BM;  // weight rows per tile
  constexpr int RO1 = MODE == 2 ? BM : 0;      // row offset of the second matrix
  const int MT = args.OUT / TR;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NA; ++i) {
      mbar_init(&a_full[i], C::Q4 ? 8 : 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < C::SP; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], 8);
    }
    for (int i = 0; i < C::SB; ++i) {
      mbar_init(&b_full[i], 32);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < C::RINGN; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    for (int i = 0; i < C::SS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 32);
      mbar_init(&t_empty[i], 8);
      mbar_init(&x_full[i], 128);
      mbar_init(&x_empty[i], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // tile plan: plan[u] = first flat n-tile of group u (prefix of ceil(count / BN))
  const int U = min(args.counts[0], args.max_groups);
  for (int u = threadIdx.x; u < U; u += blockDim.x)
    plan[u + 1] = (args.group_off[u + 1] - args.group_off[u] + BN - 1) / BN;
  if (threadIdx.x == 0) plan[0] = 0;
  __syncthreads();
  if (warp == 0) {  // inclusive scan of plan[1..U] by one warp, in 32-entry blocks
    int carry = 0;
    for (int base = 1; base <= U; base += 32) {
      const int i = base + lane;
      int v = i <= U ? plan[i] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
      }
      if (i <= U) plan[i] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int NT = plan[U];
  const int total = NT * MT;

  if (warp == 0) {
    // ---------------------------------------------------------------- weight + scale producer
    if (lane == 0) {
      // 8-bit: one A stage per K stage; 4-bit: one packed stage per two K stages
      constexpr int WR = C::Q4 ? C::SP : C::SA;
      uint64_t* wfull = C::Q4 ? p_full : a_full;
      uint64_t* wempty = C::Q4 ? p_empty : a_empty;
      int sa = 0, ss = 0, issued = 0, s_issued = 0;
      uint32_t pa = 0, sph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const ITile tl = itile_of<BN>(t, plan, U, NT, args);
        // a slot outside the arena gives negative or out-of-range rows: the
        // TMA's zero fill (the epilogue writes zeros for such tiles)
        const int row0 = (tl.slot >= 0 && tl.slot < args.num_slots) ? tl.slot * args.OUT + tl.m * TR : -TR;
        for (int ks = 0; ks < NKS && ok; ++ks) {
          if ((ks & 3) == 0) {  // scales and biases of groups [2 ks, 2 ks + 8) of the tile's rows
            ok = wait_bar(&s_empty[ss], sph ^ 1, ctl, BACKOFF_NS);
            if (!ok) break;
            uint8_t* dst = sS + ss * C::S_BYTES;
            mbar_expect_tx(&s_full[ss], C::S_BYTES);
            tma_load_2d(dst, &tmS0, 2 * ks, row0, &s_full[ss]);
            tma_load_2d(dst + BM * 16, &tmQ0, 2 * ks, row0, &s_full[ss]);
            tma_load_2d(dst + 2 * BM * 16, &tmS1, 2 * ks, row0 + RO1, &s_full[ss]);
            tma_load_2d(dst + 3 * BM * 16, &tmQ1, 2 * ks, row0 + RO1, &s_full[ss]);
            ++s_issued;
            if (++ss == C::SS) { ss = 0; sph ^= 1; }
          }
          if (C::Q4 && (ks & 1)) continue;  // this K stage came with the previous packed stage
          ok = wait_bar(&wempty[sa], pa ^ 1, ctl, BACKOFF_NS);
          if (!ok) break;
          const int col = (C::Q4 ? ks / 2 : ks) * 32;  // 32 packed words = 128 bytes of every row
          mbar_expect_tx(&wfull[sa], C::A_BYTES);
          tma_load_2d(sA + sa * C::A_BYTES, &tmA0, col, row0, &wfull[sa]);
          tma_load_2d(sA + sa * C::A_BYTES + C::A_MAT, &tmA1, col, row0 + RO1, &wfull[sa]);
          ++issued;
          if (++sa == WR) { sa = 0; pa ^= 1; }
        }
      }
      if (!ok) {  // drain this thread's copies still in flight (bounded)
        for (int i = 0; i < min(issued, WR); ++i) {
          int s = sa - 1 - i;
          uint32_t p = pa;
          if (s < 0) { s += WR; p ^= 1; }
          const long long t0 = clock64();
          while (!mbar_try_wait(&wfull[s], p) && clock64() - t0 < WAIT_CYCLES) {
          }
        }
        for (int i = 0; i < min(s_issued, C::SS); ++i) {
          int s = ss - 1 - i;
          uint32_t p = sph;
          if (s < 0) { s += C::SS; p ^= 1; }
          const long long t0 = clock64();
          while (!mbar_try_wait(&s_full[s], p) && clock64() - t0 < WAIT_CYCLES) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8<NB>();
      int sa = 0, sb = 0, gc = 0;
      uint32_t pa = 0, pb = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        for (int ks = 0; ks < NKS && ok; ++ks) {
          ok = wait_bar(&b_full[sb], pb, ctl) && wait_bar(&a_full[sa], pa, ctl);
          if (!ok) break;
          tc_fence_after();
          // (8-bit A in shared memory; 4-bit A in tensor memory, addressed below)
          const uint64_t ad0 = desc_sw128(smem_u32(sA + (C::Q4 ? 0 : sa) * C::A_BYTES));
          const uint64_t ad1 = desc_sw128(smem_u32(sA + (C::Q4 ? 0 : sa) * C::A_BYTES + C::A_MAT));
          const uint64_t bd = desc_sw128(smem_u32(sB + sb * C::B_BYTES));
#pragma unroll
          for (int gi = 0; gi < KS / GSZ; ++gi) {
            const int slot = gc % C::RINGN;
            ok = wait_bar(&acc_empty[slot], ((gc / C::RINGN) & 1) ^ 1, ctl);
            if (!ok) break;
            tc_fence_after();
            const uint32_t d = tmem + slot * C::ACC_COLS;
#pragma unroll
            for (int kk = 0; kk < GSZ / 32; ++kk) {
              // K step of 32 one-byte elements = 32 bytes: +2 in the descriptor's
              // address field, 8 columns of tensor memory
              const uint32_t ko = static_cast<uint32_t>((gi * GSZ + kk * 32) >> 4);
              if constexpr (C::Q4) {
                const uint32_t at = tmem + C::ACC_TOTAL + sa * C::A_TCOLS + (gi * GSZ + kk * 32) / 4;
                umma_i8_ts(d, at, bd + ko, idesc, kk);
                umma_i8_ts(d + NB, at + KS / 4, bd + ko, idesc, kk);
              } else {
                umma_i8(d, ad0 + ko, bd + ko, idesc, kk);
                umma_i8(d + NB, ad1 + ko, bd + ko, idesc, kk);
              }
            }
            umma_commit(&acc_full[slot]);
            ++gc;
          }
          if (!ok) break;
          umma_commit(&a_empty[sa]);
          if (++sa == NA) { sa = 0; pa ^= 1; }
          umma_commit(&b_empty[sb]);
          if (++sb == C::SB) { sb = 0; pb ^= 1; }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- piece rows + pair table
    // lane l copies chunk l % 8 of B rows l / 8 + 4 i (i < 2 BN / 4): pair
    // (l / 8 + 4 i) % BN, plane (hi / lo) (l / 8 + 4 i) / BN
    static_assert(BN == 8 || BN == 16, "8 or 16 pairs per tile");
    constexpr int RPL = BN / 4;  // pairs per lane
    const int c = lane & 7, r0 = lane >> 3;
    const size_t prow_bytes = static_cast<size_t>(2) * K;
    int sb = 0, it = 0;
    uint32_t pb = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const ITile tl = itile_of<BN>(t, plan, U, NT, args);
      // input row of pair j (lane j < BN), -1 past the tile's pairs
      int myrow = -1;
      if (lane < BN && lane < tl.nvalid) {
        const int pos = tl.goff + tl.n0 + lane;
        const int rw = args.in_by_pos ? pos : args.perm[pos] / args.pair_div;
        myrow = (rw >= 0 && rw < args.in_rows) ? rw : -1;
      }
      int row[RPL];
#pragma unroll
      for (int q = 0; q < RPL; ++q) row[q] = __shfl_sync(0xffffffffu, myrow, r0 + 4 * q);
      // the pairs' (E, X) per group, transposed to [group][E, X][pair]
      const int buf = it & 1;
      ok = wait_bar(&t_empty[buf], ((it >> 1) & 1) ^ 1, ctl, BACKOFF_NS);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      float* tp = sT + buf * (C::T_BYTES / 4);
      for (int idx = lane; idx < BN * G; idx += 32) {
        const int j = idx % BN, g = idx / BN;
        const int rw = __shfl_sync(0xffffffffu, myrow, j);
        float2 v = make_float2(0.f, 0.f);
        if (rw >= 0) v = *reinterpret_cast<const float2*>(args.ex + ((size_t)rw * G + g) * 2);
        tp[g * 2 * BN + j] = v.x;
        tp[g * 2 * BN + BN + j] = v.y;
      }
      mbar_arrive(&t_full[buf]);
      for (int ks = 0; ks < NKS; ++ks) {
        ok = wait_bar(&b_empty[sb], pb ^ 1, ctl, BACKOFF_NS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        uint8_t* dst = sB + sb * C::B_BYTES;
        const int8_t* col = args.pieces + ks * KS + c * 16;
#pragma unroll
        for (int i = 0; i < 2 * RPL; ++i) {
          const int rr = r0 + 4 * i;  // B row: pair rr % BN, plane rr / BN
          const int rw = row[i % RPL];
          const bool v = rw >= 0;
          cp_async16(dst + rr * KS + ((c ^ (rr & 7)) << 4),
                     v ? col + rw * prow_bytes + (i >= RPL ? K : 0) : args.pieces, v ? 16u : 0u);
        }
        cp_async_arrive(&b_full[sb]);
        if (++sb == C::SB) { sb = 0; pb ^= 1; }
      }
    }
    cp_async_wait_all();  // no copy of this warp outlives the kernel
  } else if (warp < C::UNP_WARP0) {
    // ---------------------------------------------------------------- epilogue: 8 warps, (quadrant, matrix)
    const int quad = warp & 3;
    const int mat = (warp - C::EPI_WARP0) >> 2;  // gate / up, or the tile's first / second 128 rows
    const int r = quad * 32 + lane;              // weight row within the tile, TMEM lane
    int ss = 0, gc = 0, it = 0;
    uint32_t sph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const ITile tl = itile_of<BN>(t, plan, U, NT, args);
      const int buf = it & 1;
      const uint32_t bph = (it >> 1) & 1;
      ok = wait_bar(&t_full[buf], bph, ctl, BACKOFF_NS);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const float* tp = sT + buf * (C::T_BYTES / 4);
      const int nq = (tl.nvalid + 3) >> 2;  // 4-pair chunks holding valid pairs (warp-uniform)
      float y[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) y[j] = 0.0f;
      for (int g8 = 0; g8 < G && ok; g8 += 8) {
        ok = wait_bar(&s_full[ss], sph, ctl, BACKOFF_NS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* sc = sS + ss * C::S_BYTES + mat * (2 * BM * 16) + r * 16;
        const uint4 sv = *reinterpret_cast<const uint4*>(sc);
        const uint4 bv = *reinterpret_cast<const uint4*>(sc + BM * 16);
        // generic reads of the chunk before the TMA (async proxy) refills it
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[ss]);
        if (++ss == C::SS) { ss = 0; sph ^= 1; }
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
        // GP groups per hand-off: both accumulators are loaded before one
        // wait, so the load latency is paid once per GP groups
        constexpr int GP = BN == 8 ? 2 : 1;
#pragma unroll
        for (int gi0 = 0; gi0 < 8; gi0 += GP) {
          int slot[GP];
#pragma unroll
          for (int p = 0; p < GP; ++p) {
            slot[p] = (gc + p) % C::RINGN;
            if (ok) ok = wait_bar(&acc_full[slot[p]], ((gc + p) / C::RINGN) & 1, ctl);
          }
          ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-wide
          if (!ok) break;
          tc_fence_after();
          uint32_t a[GP][NB];
#pragma unroll
          for (int p = 0; p < GP; ++p)
            tmem_ld_cols(tmem + (static_cast<uint32_t>(quad * 32) << 16) + slot[p] * C::ACC_COLS + mat * NB, a[p]);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int p = 0; p < GP; ++p) mbar_arrive(&acc_empty[slot[p]]);
          }
          gc += GP;
#pragma unroll
          for (int p = 0; p < GP; ++p) {
            const int gi = gi0 + p;
            const float s = (gi & 1) ? hi_bf16(sw[gi >> 1]) : lo_bf16(sw[gi >> 1]);
            const float b = (gi & 1) ? hi_bf16(bw[gi >> 1]) : lo_bf16(bw[gi >> 1]);
            const float* e = tp + (g8 + gi) * 2 * BN;
#pragma unroll
            for (int q = 0; q < BN / 4; ++q) {
              if (q < nq) {
                const float4 e4 = *reinterpret_cast<const float4*>(e + 4 * q);
                const float4 x4 = *reinterpret_cast<const float4*>(e + BN + 4 * q);
                const float ev[4] = {e4.x, e4.y, e4.z, e4.w}, xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                  const int j = 4 * q + jj;
                  // 256 * sum(q hi) + sum(q lo): |.| < 2^28, exact in int32
                  const int qi = static_cast<int>(a[p][j]) * 256 + static_cast<int>(a[p][BN + j]);
                  const float f = __int2float_rn(qi) * ev[jj];
                  y[j] = fmaf(b, xv[jj], fmaf(f, s, y[j]));
                }
              }
            }
          }
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[buf]);
      if constexpr (MODE == 2) {  // down projection: this warp's 32 output columns of the tile's pairs
        const bool slot_ok = tl.slot >= 0 && tl.slot < args.num_slots;
        int my_row = 0;
        if (lane < tl.nvalid) {
          const int pos = tl.goff + tl.n0 + lane;
          my_row = args.out_by_pos ? pos : args.perm[pos];
        }
        const int ocol = tl.m * TR + mat * BM + r;
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int orow = __shfl_sync(0xffffffffu, my_row, j);
          if (j < tl.nvalid) args.out[(size_t)orow * args.OUT + ocol] = slot_ok ? f32_to_bf16(y[j]) : 0;
        }
        continue;
      }
      // hand-off: the up warps pass their sums to the gate warps of the quadrant
      float* xr = sX + buf * (C::X_BYTES / 4) + r * C::X_STRIDE;
      if (mat == 1) {
        ok = wait_bar(&x_empty[buf], bph ^ 1, ctl, BACKOFF_NS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
#pragma unroll
        for (int q = 0; q < BN / 4; ++q)
          *reinterpret_cast<float4*>(xr + 4 * q) = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        mbar_arrive(&x_full[buf]);
      } else {
        ok = wait_bar(&x_full[buf], bph, ctl, BACKOFF_NS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        float u[BN];
#pragma unroll
        for (int q = 0; q < BN / 4; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(xr + 4 * q);
          u[4 * q] = v.x; u[4 * q + 1] = v.y; u[4 * q + 2] = v.z; u[4 * q + 3] = v.w;
        }
        mbar_arrive(&x_empty[buf]);
        const bool slot_ok = tl.slot >= 0 && tl.slot < args.num_slots;
        int my_row = 0;  // output row of pair `lane`, broadcast by shuffle
        if (lane < tl.nvalid) {
          const int pos = tl.goff + tl.n0 + lane;
          my_row = args.out_by_pos ? pos : args.perm[pos];
        }
        const int ocol = tl.m * BM + r;
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int orow = __shfl_sync(0xffffffffu, my_row, j);
          if (j < tl.nvalid)
            args.out[(size_t)orow * args.OUT + ocol] = slot_ok ? swiglu_bf16(y[j], u[j]) : 0;
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- 4-bit unpacking: 8 warps, (quadrant, matrix)
    // Each thread takes its row's 128 packed bytes of a stage into registers
    // (releasing the slot at once), then per K stage turns 64 bytes into 128:
    // word w -> (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F), nibbles 0,2,4,6 then
    // 1,3,5,7, stored as 32 tensor-memory columns of its lane.
    if constexpr (C::Q4) {
      const int quad = warp & 3;
      const int mat = (warp - C::UNP_WARP0) >> 2;
      const int r = quad * 32 + lane;
      int sp = 0, sa = 0;
      uint32_t pp = 0, pa = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        for (int ks = 0; ks < NKS && ok; ks += 2) {
          ok = wait_bar(&p_full[sp], pp, ctl);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          const uint8_t* prow = sA + sp * C::A_BYTES + mat * C::A_MAT + r * 128;
          uint4 v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = *reinterpret_cast<const uint4*>(prow + ((i ^ (r & 7)) << 4));
          // generic reads of the slot before the TMA (async proxy) refills it
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_empty[sp]);
          if (++sp == C::SP) { sp = 0; pp ^= 1; }
#pragma unroll
          for (int hs = 0; hs < 2; ++hs) {
            if (ks + hs >= NKS) break;
            ok = wait_bar(&a_empty[sa], pa ^ 1, ctl);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 w4 = v[4 * hs + c];
              const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                o[2 * (4 * c + q)] = w[q] & 0x0F0F0F0Fu;
                o[2 * (4 * c + q) + 1] = (w[q] >> 4) & 0x0F0F0F0Fu;
              }
            }
            tc_fence_after();
            tmem_st32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + C::ACC_TOTAL + sa * C::A_TCOLS + mat * (KS / 4),
                      o);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[sa]);
            if (++sa == C::SAT) { sa = 0; pa ^= 1; }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ------------------------------------------------------------------ host side
// Whether the integer-operand gate/up serves this arena: 8-bit affine weights,
// K a multiple of 128 with at most 64 groups (whole scale chunks of 8 groups),
// 128-row output tiles.
static bool supported(const sg_arena* A, bool dual, int grid_groups) {
  const int K = dual ? A->hidden : A->inter, OUT = dual ? A->inter : A->hidden;
  // 4-bit stages hold two K stages each; whole scale chunks of 8 groups
  return (A->bits == 8 || A->bits == 4) && A->group_size == GSZ && K % (A->bits == 4 ? 2 * KS : KS) == 0 &&
         (K / GSZ) % 8 == 0 && K / GSZ <= Cfg<8, 16>::GMAX && OUT % (dual ? BM : 2 * BM) == 0 &&
         grid_groups <= PLAN_MAX_GROUPS;
}

template <int BITS, int MODE, int BN>
static int launch(const sg_arena* A, const Args& args, cudaStream_t s) {
  using C = Cfg<BITS, BN>;
  constexpr bool DUAL = MODE == 1;
  const int K = args.K;
  const uint64_t rows_total = (uint64_t)A->num_slots * args.OUT;
  const uint64_t words = (uint64_t)K * BITS / 32;
  const uint64_t groups = (uint64_t)K / GSZ;
  const void* w0 = DUAL ? A->gate_w : A->down_w;
  const void* w1 = DUAL ? A->up_w : A->down_w;
  const void* s0 = DUAL ? A->gate_s : A->down_s;
  const void* b0 = DUAL ? A->gate_b : A->down_b;
  const void* s1 = DUAL ? A->up_s : A->down_s;
  const void* b1 = DUAL ? A->up_b : A->down_b;
  CUtensorMap m0, m1, ms0, mq0, ms1, mq1;
  const bool ok =
      make_map(&m0, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w0, words, rows_total, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
      make_map(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w1, words, rows_total, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
      make_map(&ms0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s0, groups, rows_total, 8, BM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
      make_map(&mq0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b0, groups, rows_total, 8, BM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
      make_map(&ms1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s1, groups, rows_total, 8, BM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
      make_map(&mq1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b1, groups, rows_total, 8, BM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return SG_ERR_CUDA;
  static bool attr_done[64] = {};  // per device
  int dev = 0;
  SG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
  if (!attr_done[dev]) {
    SG_CUDA_TRY(cudaFuncSetAttribute(glu_i8_kernel<BITS, MODE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM));
    attr_done[dev] = true;
  }
  glu_i8_kernel<BITS, MODE, BN><<<num_sms(), C::THREADS, C::SMEM, s>>>(m0, m1, ms0, mq0, ms1, mq1, args);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

}  // namespace i8

// Pieces of `rows` rows of K bf16 values (see sg_quantize_pieces); with
// perm, of the rows the pair positions use, in dispatch order (above).
int quantize_pieces(const uint16_t* x, int rows, int K, int order, int8_t* pieces, float* ex, cudaStream_t s,
                    const int32_t* perm, int pair_div, int in_pos, const int32_t* counts,
                    const int32_t* group_off) {
  if (rows == 0) return SG_OK;
  const long long chunks = (long long)rows * (K / 8);
  const long long blocks = (chunks + 255) / 256;
  if (blocks > 0x7FFFFFFFLL) return SG_ERR_SHAPE;
  i8::quantize_pieces_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, rows, K, order, pieces, ex, perm,
                                                                           pair_div, in_pos, counts, group_off);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

bool i8_supported(const sg_arena* A, bool dual, int grid_groups) { return i8::supported(A, dual, grid_groups); }

// Pair-tile width of the integer-operand kernels: 8 (twice the accumulators
// in flight, half the epilogue per group) while groups average at most
// i8::TILE8_MAX pairs, else 16; sg_set_glu_tile forces one.
static int g_i8_tile = 0;
int i8_tile_width(int num_pairs, int grid_groups) {
  if (g_i8_tile) return g_i8_tile;
  const int avg = (num_pairs + grid_groups - 1) / (grid_groups > 0 ? grid_groups : 1);
  return avg <= i8::TILE8_MAX ? 8 : 16;
}
// 0 automatic; 8 fixes the integer-operand kernels' tile, 32/64/128 the
// dequantising kernels', 16 both.
int set_i8_tile(int bn) {
  if (bn != 0 && bn != 8 && bn != 16 && bn != 32 && bn != 64 && bn != 128) return SG_ERR_INVALID_ARG;
  g_i8_tile = bn <= 16 ? bn : 0;
  g_tc_tile = bn >= 16 ? bn : 0;
  return SG_OK;
}

// dual: gate/up + SwiGLU (K = hidden, OUT = inter); else the down projection
// (K = inter, OUT = hidden).
int i8_glu_launch(const sg_arena* A, bool dual, const int8_t* pieces, const float* ex, int in_rows, int pair_div,
                  int in_by_pos, int out_by_pos, const int32_t* counts, const int32_t* slot_ids,
                  const int32_t* group_off, const int32_t* perm, int grid_groups, int num_pairs, uint16_t* out,
                  cudaStream_t s) {
  i8::Args a;
  a.num_slots = A->num_slots;
  a.K = dual ? A->hidden : A->inter;
  a.OUT = dual ? A->inter : A->hidden;
  a.pieces = pieces;
  a.ex = ex;
  a.in_rows = in_rows;
  a.counts = counts;
  a.slot_ids = slot_ids;
  a.group_off = group_off;
  a.perm = perm;
  a.pair_div = pair_div;
  a.in_by_pos = in_by_pos;
  a.out_by_pos = out_by_pos;
  a.max_groups = grid_groups;
  a.out = out;
  const int bn = i8_tile_width(num_pairs, grid_groups);
  if (bn == 8) {
    if (A->bits == 4) return dual ? i8::launch<4, 1, 8>(A, a, s) : i8::launch<4, 2, 8>(A, a, s);
    return dual ? i8::launch<8, 1, 8>(A, a, s) : i8::launch<8, 2, 8>(A, a, s);
  }
  if (A->bits == 4) return dual ? i8::launch<4, 1, 16>(A, a, s) : i8::launch<4, 2, 16>(A, a, s);
  return dual ? i8::launch<8, 1, 16>(A, a, s) : i8::launch<8, 2, 16>(A, a, s);
}

}  // namespace sg
