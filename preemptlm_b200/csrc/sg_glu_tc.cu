// Gathered SwiGLU expert matmuls on the 5th-generation tensor cores (tcgen05 +
// TMEM), fed by TMA, for the slot arena (a9, a10, a12).
//
// Tile = (group u, 128 weight rows of one projection, BN pairs of u).  The
// weight tile is the MMA's A operand (M = 128 rows, K-major), the pairs' input
// rows are B (N = BN, K-major), the fp32 accumulator D[128 x BN] lives in
// TMEM.  gate/up run as two MMAs into two accumulators and the epilogue forms
// SwiGLU; the down projection has one.  Accumulators are double buffered so
// the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Warp roles (15 warps, one CTA per SM, persistent over a static tile list):
//   w0      TMA producer of weight tiles: bf16 straight into the SW128 operand
//           layout, or packed 8/4-bit words (128 bytes per row, SW128) for the
//           dequantisers
//   w1      TMEM allocation + single-thread tcgen05.mma issue + commits
//   w2      TMA gather4 producer of the B rows (token rows picked by the
//           dispatch permutation) into its own ring
//   w3-w10  dequantisers (quantised arenas): 256 threads, each one row of one
//           matrix (gate/up) or half a row (down); w = bf16(scale * q + bias)
//           computed exactly in fp32 with magic-number integer-to-float and
//           packed f32x2 FMA/ADD, written in the SW128 operand layout
//   w11-w14 epilogue: tcgen05.ld -> SwiGLU / bf16 -> global, one warp per
//           32-lane TMEM quadrant
//
// Every mbarrier wait is bounded (about one second of clock64); on expiry the
// CTA records SG_ERR_TIMEOUT in the library's device status word, drains the
// copies it issued (bounded as well), frees its TMEM and returns.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "sg_common.cuh"

namespace sg {

__device__ int g_device_status = 0;  // first error recorded by a kernel of this library

namespace tc {

constexpr int BM = 128;            // weight rows per tile (MMA M)
constexpr int BK = 64;             // K per pipeline stage (one 128-byte swizzle atom of bf16)
constexpr int DQ_WARP0 = 3;  // dequantiser warps start here; the 4 epilogue warps follow them
constexpr int RING_BUDGET = 208 * 1024;
constexpr int PLAN_MAX_GROUPS = 2048;
constexpr long long WAIT_CYCLES = 2000000000LL;  // ~1 s
constexpr uint32_t BACKOFF_NS = 512;

__host__ __device__ constexpr int pow2ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

// MODE 0: down projection, one 128-row weight tile; 1: gate/up, two matrices
// and the SwiGLU epilogue; 2: down projection, two 128-row halves of a 256-row
// weight tile sharing the B rows (twice the bytes per pipeline stage).
template <int BITS, int MODE, int BN>
struct Cfg {
  static constexpr bool DUAL = MODE != 0;  // two A matrices per stage
  static constexpr int ROWS = MODE == 2 ? 2 * BM : BM;  // weight rows per tile
  static constexpr int NMAT = DUAL ? 2 : 1;
  // ATM: dequantised A tiles live in tensor memory (tcgen05.st by the
  // dequantisers, read by tcgen05.mma), sparing shared-memory bandwidth;
  // used for quantised arenas at decode tile widths
  static constexpr bool ATM = BITS != 16 && BN <= 64;
  static constexpr int A_MAT = BM * BK * 2;                       // one bf16 operand tile
  static constexpr int A_BYTES = ATM ? 0 : NMAT * A_MAT;          // shared-memory A stage
  // one packed tile: 128 rows x 128 bytes (KP operand stages of BK weights)
  static constexpr int KP = BITS == 16 ? 1 : 128 * 8 / (BK * BITS);
  static constexpr int P_MAT = BITS == 16 ? 0 : BM * 128;
  static constexpr int P_BYTES = NMAT * P_MAT;
  static constexpr int B_SUB = BN * BK * 2;  // one operand stage of B (BN rows x BK)
  // B stages span KBB operand stages and run SB deep, so the row gathers are
  // issued well ahead of the MMAs (they queue in the SM's TMA unit behind the
  // weight loads)
  static constexpr int KBB = BN <= 32 ? 4 : (BN <= 64 ? 2 : 1);
  static constexpr int B_BYTES = B_SUB * KBB;
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int NACC = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int ACC_TOTAL = NACC * ACC_COLS;
  static constexpr int A_TCOLS = NMAT * BK / 2;  // TMEM columns of one A stage (two bf16 per column)
  static constexpr int SB = cmin(6, cmax(2, 49152 / B_BYTES));
  static constexpr int SA = ATM ? cmin(6, (512 - ACC_TOTAL) / A_TCOLS)
                                : cmin(BITS == 16 ? 8 : 3, (RING_BUDGET - SB * B_BYTES -
                                                            (BITS == 16 ? 0 : 2 * NMAT * BM * 128)) / A_BYTES);
  // packed ring: deep enough to cover HBM latency (~1 us at 96 KB per SM in
  // flight), shallow enough that the B gathers queued behind it in the SM's
  // TMA unit still land ahead of the MMAs
  static constexpr int SP = BITS == 16 ? 0
                          : cmin(ATM ? (DUAL ? 3 : 4) : 6, (RING_BUDGET - SA * A_BYTES - SB * B_BYTES) / P_BYTES);
  static constexpr int TMEM_USED = ACC_TOTAL + (ATM ? SA * A_TCOLS : 0);
  // operand stages per MMA-side wait on a_full: TMA-filled stages may land out
  // of order and are waited one by one
  static constexpr int MG = (BITS != 16 && SA >= 4) ? 2 : 1;
  static constexpr int TMEM_COLS = pow2ceil(TMEM_USED < 32 ? 32 : TMEM_USED);
  // shared memory carve-up (offsets from a 1024-aligned base)
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + SA * A_BYTES;
  static constexpr int OFF_P = OFF_B + SB * B_BYTES;
  static constexpr int OFF_PLAN = OFF_P + SP * P_BYTES;
  // ATM configs also keep the groups' offsets and slots in shared memory, so
  // that finding a tile's rows never waits on a global load
  static constexpr bool TILE_SMEM = ATM;
  static constexpr int OFF_TILE = OFF_PLAN + (PLAN_MAX_GROUPS + 1) * 4;
  // ATM configs stage scale/bias rows by TMA (when the group count is a
  // multiple of 8): a chunk is 8 groups (16 bytes) x 128 rows per array,
  // arrays [matrix][scales, biases], SS chunks in flight
  static constexpr int SS = ATM ? 3 : 0;
  static constexpr int S_BYTES = NMAT * 2 * BM * 16;
  static constexpr int OFF_S = (OFF_TILE + (TILE_SMEM ? (2 * PLAN_MAX_GROUPS + 1) * 4 : 0) + 127) & ~127;
  static constexpr int OFF_BAR = (OFF_S + SS * S_BYTES + 15) & ~15;
  static constexpr int NUM_BARS = 2 * SA + 2 * SB + 2 * SP + 2 * NACC + 2 * SS;
  static constexpr int SMEM = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + tmem slot/abort flag + align slack
  // dequantiser warps: 8, each thread one row of one matrix (gate / up), or
  // half a row of the single matrix (down); one TMEM lane quadrant per warp
  static constexpr int DQW = BITS == 16 ? 0 : 8;
  static constexpr int EPI_WARP0 = DQ_WARP0 + DQW;
  static constexpr int THREADS = (EPI_WARP0 + 4) * 32;
  static_assert(SA >= 2 && (BITS == 16 || SP >= 2), "pipeline too shallow");
  static_assert(TMEM_COLS <= 512, "tensor memory budget");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(B_SUB % 1024 == 0, "B tile must keep 1024-byte alignment");
};

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.b32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As above, but a thread whose phase is not complete is suspended until it
// completes or about `ns` nanoseconds pass, instead of spinning on issue slots
// that the dequantising warps of its SM sub-partition need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.b32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

struct Ctl {
  volatile int* abort;  // shared flag: a wait in this CTA expired
};

// Bounded wait for the phase of parity `parity` to complete.
// Roles off the critical path (producers, epilogue) back off with a short
// nanosleep between polls, leaving issue slots to the dequantising warps that
// share their SM sub-partition.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctl ctl, uint32_t backoff_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 200000)) return true;  // wakes on completion
    if (backoff_ns) __nanosleep(backoff_ns);
    if (*ctl.abort) return false;
    if (clock64() - t0 > WAIT_CYCLES) {
      *ctl.abort = 1;
      atomicCAS(&g_device_status, 0, SG_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
// 16-byte LSU copy global -> shared (zero fill when src_bytes == 0); completion
// is tracked per thread and reported to an mbarrier by cp_async_arrive.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
// One arrival on `bar` once every cp.async this thread issued so far has landed
// (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Bring [p, p + bytes) into L2 (16-byte aligned address and size).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;              // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;      // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;              // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;              // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// A from tensor memory (K-major, row m in lane m, two bf16 of consecutive k per column)
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ dequantisation
// w = fp32(scale * q + bias), exactly as the oracle forms it, then bf16:
//   v = 2^15 + q * 2^(p - 8) is built by placing q at bit p of the mantissa of
//   2^15 (one PRMT / LOP3; the field must end below bit 23, the exponent);
//   fma(v, s_p, -2^15 * s_p) = q * scale exactly (s_p = scale * 2^(8 - p), a
//   power-of-two rescale); then one add of bias.
// Fused form: when c_p = bias - 2^15 * s_p is exact in fp32 (checked per group
// with an error-free two-sum), fma(v, s_p, c_p) rounds the exact scale*q + bias
// once -- the same value as fp32(scale * q) + bias, since scale * q (8 + 8
// significant bits) is exact -- in one instruction instead of two.
// Two weights at a time with packed fma.rn.f32x2 / add.rn.f32x2.
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
template <bool FUSED>
__device__ __forceinline__ uint32_t dq_pair(uint32_t v_lo, uint32_t v_hi, unsigned long long s2,
                                            unsigned long long c2, unsigned long long b2) {
  const unsigned long long v = (static_cast<unsigned long long>(v_hi) << 32) | v_lo;
  unsigned long long t, w;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(t) : "l"(v), "l"(s2), "l"(c2));
  if (FUSED) w = t;
  else asm("add.rn.f32x2 %0, %1, %2;" : "=l"(w) : "l"(t), "l"(b2));
  __nv_bfloat162 r = __floats2bfloat162_rn(__uint_as_float(static_cast<uint32_t>(w)),
                                           __uint_as_float(static_cast<uint32_t>(w >> 32)));
  return *reinterpret_cast<uint32_t*>(&r);
}

struct GroupScale {  // one (scale, bias) group in the forms the converters use
  // q8: p1 = (s, s).  q4: p1 = (s8, s12), p2 = (s16, s8), p3 = (s12, s16) with
  // s_p = scale * 2^(8 - p); c* = k - 2^15 * s* with k = bias when the warp
  // runs fused, else 0; b = (bias, bias)
  unsigned long long p1, c1, p2, c2, p3, c3, b;
  bool fused;  // warp-uniform
};
// b - x, and whether that difference is exact in fp32 (Knuth's two-sum error is zero)
__device__ __forceinline__ float sub_exact(float b, float x, bool& exact) {
  const float d = __fsub_rn(b, x);
  const float bv = __fsub_rn(d, b);
  const float err = __fadd_rn(__fsub_rn(b, __fsub_rn(d, bv)), __fsub_rn(-x, bv));
  exact = exact && err == 0.0f;
  return d;
}
template <int BITS>
__device__ __forceinline__ GroupScale make_scale(float s, float b) {
  GroupScale g;
  g.b = f2pack(b, b);
  bool ex = true;
  if (BITS == 8) {
    const float x = 32768.0f * s;
    const float cf = sub_exact(b, x, ex);
    g.fused = __all_sync(0xffffffffu, ex);
    g.p1 = f2pack(s, s);
    g.c1 = g.fused ? f2pack(cf, cf) : f2pack(-x, -x);
  } else {
    const float s8 = s, s12 = s * 0.0625f, s16 = s * 0.00390625f;
    const float x8 = 32768.0f * s8, x12 = 32768.0f * s12, x16 = 32768.0f * s16;
    const float f8 = sub_exact(b, x8, ex), f12 = sub_exact(b, x12, ex), f16 = sub_exact(b, x16, ex);
    g.fused = __all_sync(0xffffffffu, ex);
    g.p1 = f2pack(s8, s12);
    g.p2 = f2pack(s16, s8);
    g.p3 = f2pack(s12, s16);
    if (g.fused) {
      g.c1 = f2pack(f8, f12);
      g.c2 = f2pack(f16, f8);
      g.c3 = f2pack(f12, f16);
    } else {
      g.c1 = f2pack(-x8, -x12);
      g.c2 = f2pack(-x16, -x8);
      g.c3 = f2pack(-x12, -x16);
    }
  }
  return g;
}

// q8: 16-byte packed chunk (16 weights) -> two 16-byte bf16 chunks
template <bool FUSED>
__device__ __forceinline__ void dq8_chunk(uint4 v, const GroupScale& g, uint4& o0, uint4& o1) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a0 = __byte_perm(w[i], 0x47000000u, 0x7404);
    const uint32_t a1 = __byte_perm(w[i], 0x47000000u, 0x7414);
    const uint32_t a2 = __byte_perm(w[i], 0x47000000u, 0x7424);
    const uint32_t a3 = __byte_perm(w[i], 0x47000000u, 0x7434);
    o[2 * i] = dq_pair<FUSED>(a0, a1, g.p1, g.c1, g.b);
    o[2 * i + 1] = dq_pair<FUSED>(a2, a3, g.p1, g.c1, g.b);
  }
  o0 = make_uint4(o[0], o[1], o[2], o[3]);
  o1 = make_uint4(o[4], o[5], o[6], o[7]);
}

// q4: one packed word (8 weights, nibble m at bits 4m) -> one 16-byte bf16 chunk.
// A nibble may sit at mantissa bit 8, 12 or 16 only (bits 20-23 would reach
// the exponent), so three shifted copies of the word feed the eight weights.
template <bool FUSED>
__device__ __forceinline__ uint4 dq4_word(uint32_t w, const GroupScale& g) {
  const uint32_t a = w << 8, b = w >> 4, c = w >> 16;
  const uint32_t M = 0x47000000u;
  const uint32_t v0 = (a & 0x00000F00u) | M, v1 = (a & 0x0000F000u) | M;  // nibbles 0,1 at bits 8,12
  const uint32_t v2 = (a & 0x000F0000u) | M, v3 = (b & 0x00000F00u) | M;  // nibbles 2,3 at bits 16,8
  const uint32_t v4 = (b & 0x0000F000u) | M, v5 = (b & 0x000F0000u) | M;  // nibbles 4,5 at bits 12,16
  const uint32_t v6 = (c & 0x00000F00u) | M, v7 = (c & 0x0000F000u) | M;  // nibbles 6,7 at bits 8,12
  return make_uint4(dq_pair<FUSED>(v0, v1, g.p1, g.c1, g.b), dq_pair<FUSED>(v2, v3, g.p2, g.c2, g.b),
                    dq_pair<FUSED>(v4, v5, g.p3, g.c3, g.b), dq_pair<FUSED>(v6, v7, g.p1, g.c1, g.b));
}

// A thread's share of one packed stage, held in registers: q8 DUAL 8 chunks
// (its full 128-byte row), otherwise 4 chunks (its half of every sub-stage).
// Packed tile layout: SW128, 128-byte rows, 16-byte chunk c of row r at c ^ (r & 7).
template <int BITS, bool FULL>
__device__ __forceinline__ void load_packed(const uint8_t* p_tile, int r, int part, uint4 (&v)[8]) {
  const uint8_t* prow = p_tile + r * 128;
#pragma unroll
  for (int i = 0; i < (FULL ? 8 : 4); ++i) {
    // full row: chunk i.  Half rows: q8 sub-stage j = i / 2 uses chunks 4j + 2 part + (i & 1);
    // q4 sub-stage j = i uses chunk 2j + part.
    const int c = FULL ? i : (BITS == 8 ? 4 * (i >> 1) + 2 * part + (i & 1) : 2 * i + part);
    v[i] = *reinterpret_cast<const uint4*>(prow + ((c ^ (r & 7)) << 4));
  }
}

// Operand sub-stage j (BK weights of row r) from the register share into
// registers: out[4 k .. 4 k + 3] = output chunk k of this thread (8 bf16 each;
// FULL: the row's 8 chunks, half rows: chunks 4 part .. 4 part + 3).
template <int BITS, bool FULL, bool FUSED>
__device__ __forceinline__ void dequant_sub_regs(const uint4 (&v)[8], int j, const GroupScale& g,
                                                 uint32_t (&out)[32]) {
  if (BITS == 8) {
#pragma unroll
    for (int q = 0; q < (FULL ? 4 : 2); ++q) {
      uint4 o0, o1;
      dq8_chunk<FUSED>(v[FULL ? 4 * j + q : 2 * j + q], g, o0, o1);
      out[8 * q + 0] = o0.x; out[8 * q + 1] = o0.y; out[8 * q + 2] = o0.z; out[8 * q + 3] = o0.w;
      out[8 * q + 4] = o1.x; out[8 * q + 5] = o1.y; out[8 * q + 6] = o1.z; out[8 * q + 7] = o1.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < (FULL ? 2 : 1); ++q) {
      const uint4 pv = FULL ? v[2 * j + q] : v[j];
      const uint32_t w[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint4 o = dq4_word<FUSED>(w[h], g);
        out[16 * q + 4 * h + 0] = o.x; out[16 * q + 4 * h + 1] = o.y;
        out[16 * q + 4 * h + 2] = o.z; out[16 * q + 4 * h + 3] = o.w;
      }
    }
  }
}

// Operand sub-stage j (BK weights of row r) from the register share into the
// SW128 bf16 tile.  FULL: all 8 output chunks; half rows: chunks 4 part .. +3.
template <int BITS, bool FULL, bool FUSED>
__device__ __forceinline__ void dequant_sub(const uint4 (&v)[8], int j, uint8_t* a_tile, int r, int part,
                                            const GroupScale& g) {
  uint8_t* arow = a_tile + r * 128;
  if (BITS == 8) {
    // q8: a packed chunk = 16 weights = 2 output chunks; sub-stage j = packed chunks 4j .. 4j+3
#pragma unroll
    for (int q = 0; q < (FULL ? 4 : 2); ++q) {
      const int pc = FULL ? 4 * j + q : 2 * j + q;   // index into v
      const int oc = FULL ? 2 * q : 4 * part + 2 * q;  // first output chunk
      uint4 o0, o1;
      dq8_chunk<FUSED>(v[pc], g, o0, o1);
      *reinterpret_cast<uint4*>(arow + ((oc ^ (r & 7)) << 4)) = o0;
      *reinterpret_cast<uint4*>(arow + (((oc + 1) ^ (r & 7)) << 4)) = o1;
    }
  } else {
    // q4: a packed chunk = 32 weights = 4 output chunks; sub-stage j = packed chunks 2j, 2j+1
#pragma unroll
    for (int q = 0; q < (FULL ? 2 : 1); ++q) {
      const uint4 pv = FULL ? v[2 * j + q] : v[j];
      const uint32_t w[4] = {pv.x, pv.y, pv.z, pv.w};
      const int oc0 = FULL ? 4 * q : 4 * part;
#pragma unroll
      for (int h = 0; h < 4; ++h)
        *reinterpret_cast<uint4*>(arow + (((oc0 + h) ^ (r & 7)) << 4)) = dq4_word<FUSED>(w[h], g);
    }
  }
}

// ------------------------------------------------------------------ arguments
struct Args {
  int num_slots, K, OUT;
  const uint8_t* in;  // B rows: [in_rows, K] bf16
  int in_rows;
  const uint16_t* s0;
  const uint16_t* b0;
  const uint16_t* s1;
  const uint16_t* b1;
  const int32_t* counts;
  const int32_t* slot_ids;
  const int32_t* group_off;
  const int32_t* perm;
  int pair_div;    // B row of pair position pos: perm[pos] / pair_div, or pos when in_by_pos
  int in_by_pos;
  int out_by_pos;  // output row: pos, or perm[pos]
  int max_groups;
  uint16_t* out;
  // dense mode (dense_rows > 0): one group of dense_rows rows through slot
  // dense_slot, B row = output row = position; counts / slot_ids / group_off /
  // perm are not read.  B tiles are then contiguous rows, loaded by TMA.
  int dense_rows, dense_slot;
};

struct Tile {
  int u, m, n0, nvalid, slot, goff;
};

template <int BN>
__device__ __forceinline__ Tile tile_of(int t, const int* plan, int U, int NT, const Args& a, const int* goff_tab,
                                       const int* slot_tab) {
  Tile tl;
  tl.m = t / NT;
  const int fn = t - tl.m * NT;
  int lo = 0, hi = U;  // largest u with plan[u] <= fn
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (plan[mid] <= fn) lo = mid;
    else hi = mid;
  }
  tl.u = lo;
  tl.n0 = (fn - plan[lo]) * BN;
  if (a.dense_rows > 0) {
    tl.goff = 0;
    tl.nvalid = min(BN, a.dense_rows - tl.n0);
    tl.slot = a.dense_slot;
    return tl;
  }
  tl.goff = goff_tab[lo];
  const int cnt = goff_tab[lo + 1] - tl.goff;
  tl.nvalid = min(BN, cnt - tl.n0);
  tl.slot = slot_tab[lo];
  return tl;
}

// ------------------------------------------------------------------ the kernel
// Scale/bias stream of one dequantiser thread: V groups per vector load
// (V = 4 when the group count allows 8-byte loads, else 1), the next vector
// always in flight, crossing into the next tile of the thread's walk.
template <int V>
struct ScaleVec;
template <>
struct ScaleVec<4> {
  uint2 s, b;
  __device__ __forceinline__ void load(const uint16_t* sp, const uint16_t* bp, int v) {
    s = __ldg(reinterpret_cast<const uint2*>(sp) + v);
    b = __ldg(reinterpret_cast<const uint2*>(bp) + v);
  }
  __device__ __forceinline__ float sc(int j) const {
    const uint32_t w = j < 2 ? s.x : s.y;
    return (j & 1) ? hi_bf16(w) : lo_bf16(w);
  }
  __device__ __forceinline__ float bi(int j) const {
    const uint32_t w = j < 2 ? b.x : b.y;
    return (j & 1) ? hi_bf16(w) : lo_bf16(w);
  }
};
template <>
struct ScaleVec<1> {
  uint16_t s, b;
  __device__ __forceinline__ void load(const uint16_t* sp, const uint16_t* bp, int v) {
    s = __ldg(sp + v);
    b = __ldg(bp + v);
  }
  __device__ __forceinline__ float sc(int) const { return bf16_to_f32(s); }
  __device__ __forceinline__ float bi(int) const { return bf16_to_f32(b); }
};

// STMA: scales and biases come from the TMA-staged chunk ring in shared
// memory (8 groups per chunk) instead of per-thread global loads.
template <int BITS, int MODE, int BN, int V, bool STMA>
__device__ __forceinline__ void dequant_role(const Args& args, const int* plan, int U, int NT, int total,
                                             uint8_t* sA, const uint8_t* sP, uint64_t* a_full, uint64_t* a_empty,
                                             uint64_t* p_full, uint64_t* p_empty, Ctl ctl, uint32_t tmem_a,
                                             const int* gtab, const int* stab, const uint8_t* sS,
                                             uint64_t* s_full, uint64_t* s_empty) {
  using C = Cfg<BITS, MODE, BN>;
  constexpr bool DUAL = C::DUAL;
  // row r = 32 (warp % 4) + lane: the TMEM lane quadrant this warp may write
  const int warp = threadIdx.x >> 5;
  const int r = 32 * (warp & 3) + (threadIdx.x & 31);
  const int part = (warp - DQ_WARP0) >> 2;  // DUAL: matrix (gate / up); single: half row
  const int mat = DUAL ? part : 0;
  const int K = args.K, NKB = K / BK, groups = K / 64, nvec = groups / V;
  const uint16_t* sbase = mat ? args.s1 : args.s0;
  const uint16_t* bbase = mat ? args.b1 : args.b0;
  // per-thread row pointers of a tile (a slot outside the arena reads row 0 and
  // dequantises zeros: its A tile is the TMA's zero fill and the epilogue
  // writes zeros for it)
  auto row_ptrs = [&](int t, const uint16_t*& sp, const uint16_t*& bp, bool& sok) {
    const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
    sok = tl.slot >= 0 && tl.slot < args.num_slots;
    const size_t row = sok ? (size_t)tl.slot * args.OUT + tl.m * C::ROWS + (MODE == 2 ? mat * BM : 0) + r : 0;
    sp = sbase + row * groups;
    bp = bbase + row * groups;
  };
  int sa = 0, sp_i = 0, ss = 0;
  uint32_t pa = 0, pp = 0, sph = 0;
  bool ok = true;
  int t = blockIdx.x;
  if (t >= total) return;
  ScaleVec<V> cur, nxt;
  if constexpr (!STMA) {
    const uint16_t *cs, *cb;
    bool csok;
    row_ptrs(t, cs, cb, csok);
    cur.load(cs, cb, 0);
    int nxt_t = t, nxt_v = 1;  // (tile, vector) held in nxt
    if (nvec == 1) {
      nxt_t = t + gridDim.x;
      nxt_v = 0;
    }
    if (nxt_t < total) {
      const uint16_t *ns, *nb;
      bool nsok;
      row_ptrs(nxt_t, ns, nb, nsok);
      nxt.load(ns, nb, nxt_v);
    }
  }
  for (; t < total && ok; t += gridDim.x) {
    bool sok;
    if constexpr (STMA) {
      const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
      sok = tl.slot >= 0 && tl.slot < args.num_slots;
    } else {
      const uint16_t *tsp, *tbp;
      row_ptrs(t, tsp, tbp, sok);
    }
    uint4 pk[8];
    for (int kb0 = 0; kb0 < NKB && ok; kb0 += C::KP) {
      // take this thread's share of the packed stage into registers and
      // release the slot at once, so the producer can refill it
      ok = wait_bar(&p_full[sp_i], pp, ctl);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      load_packed<BITS, DUAL>(sP + sp_i * C::P_BYTES + mat * C::P_MAT, r, part, pk);
      // these generic-proxy reads must be ordered before the TMA (async
      // proxy) that refills the slot once it is released
      fence_async_smem();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&p_empty[sp_i]);
      if (++sp_i == C::SP) { sp_i = 0; pp ^= 1; }
      const int nsub = min(C::KP, NKB - kb0);
#pragma unroll
      for (int jp = 0; jp < C::KP; ++jp) {  // operand sub-stages (compile-time index into pk)
        const int kb = kb0 + jp;
        if (kb >= NKB) break;
        if (jp % C::MG == 0) {
          // the MMAs free operand slots in order: waiting for the last slot of
          // the next MG sub-stages covers all of them
          int sl = sa + min(C::MG, nsub - jp) - 1;
          uint32_t ph = pa;
          if (sl >= C::SA) { sl -= C::SA; ph ^= 1; }
          ok = wait_bar(&a_empty[sl], ph ^ 1, ctl);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
        }
        float gs, gb;  // this sub-stage's scale and bias
        if constexpr (STMA) {
          if ((kb & 7) == 0) {
            ok = wait_bar(&s_full[ss], sph, ctl);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
          }
          const uint8_t* sc = sS + ss * C::S_BYTES + mat * (2 * BM * 16) + r * 16 + (kb & 7) * 2;
          gs = bf16_to_f32(*reinterpret_cast<const uint16_t*>(sc));
          gb = bf16_to_f32(*reinterpret_cast<const uint16_t*>(sc + BM * 16));
          if ((kb & 7) == 7) {  // chunk done (group counts are multiples of 8 here)
            fence_async_smem();  // as for the packed slots: reads before the refilling TMA
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(&s_empty[ss]);
            if (++ss == C::SS) { ss = 0; sph ^= 1; }
          }
        } else {
          const int j = kb % V;
          if (j == 0 && kb > 0) {  // next vector of this tile becomes current
            cur = nxt;
            int vn = kb / V + 1;
            int tn = t;
            if (vn >= nvec) {
              vn = 0;
              tn = t + gridDim.x;
            }
            if (tn < total) {
              const uint16_t *ns, *nb;
              bool nsok;
              row_ptrs(tn, ns, nb, nsok);
              nxt.load(ns, nb, vn);
            }
          }
          gs = cur.sc(j);
          gb = cur.bi(j);
        }
        const GroupScale g = make_scale<BITS>(sok ? gs : 0.f, sok ? gb : 0.f);
        if (C::ATM) {
          uint32_t out[32];
          if (g.fused) dequant_sub_regs<BITS, DUAL, true>(pk, jp, g, out);
          else dequant_sub_regs<BITS, DUAL, false>(pk, jp, g, out);
          tc_fence_after();
          const uint32_t ta = tmem_a + (static_cast<uint32_t>(32 * (warp & 3)) << 16) +
                              C::ACC_TOTAL + (sa * C::NMAT + mat) * (BK / 2) + (DUAL ? 0 : 16 * part);
          if (DUAL) {  // the row's 32 columns of this stage in one store
            tmem_st32(ta, out);
          } else {
            const uint32_t (&lo)[16] = *reinterpret_cast<const uint32_t(*)[16]>(&out[0]);
            tmem_st16(ta, lo);
          }
          // one store wait per group of MG stages (the MMA reads a group only
          // once all of it is full): the first stage's stores complete while
          // the next one is computed
          if (jp % C::MG == C::MG - 1 || jp == nsub - 1) {
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) {
              for (int q = jp % C::MG; q >= 0; --q) mbar_arrive(&a_full[sa >= q ? sa - q : sa - q + C::SA]);
            }
          }
        } else {
          if (g.fused) dequant_sub<BITS, DUAL, true>(pk, jp, sA + sa * C::A_BYTES + mat * C::A_MAT, r, part, g);
          else dequant_sub<BITS, DUAL, false>(pk, jp, sA + sa * C::A_BYTES + mat * C::A_MAT, r, part, g);
          fence_async_smem();
          __syncwarp();
          if ((threadIdx.x & 31) == 0) mbar_arrive(&a_full[sa]);
        }
        if (++sa == C::SA) { sa = 0; pa ^= 1; }
      }
    }
    // the first vector of the next tile is already in nxt
    if constexpr (STMA) {
    } else if (nvec > 1 || V == 1) {
      cur = nxt;
      const int tn = t + gridDim.x;
      if (tn < total) {
        int vn = 1, tt = tn;
        if (nvec == 1) {
          vn = 0;
          tt = tn + gridDim.x;
        }
        if (tt < total) {
          const uint16_t *ns, *nb;
          bool nsok;
          row_ptrs(tt, ns, nb, nsok);
          nxt.load(ns, nb, vn);
        }
      }
    } else {
      cur = nxt;
      const int tt = t + 2 * gridDim.x;
      if (tt < total) {
        const uint16_t *ns, *nb;
        bool nsok;
        row_ptrs(tt, ns, nb, nsok);
        nxt.load(ns, nb, 0);
      }
    }
  }
}

template <int BITS, int MODE, int BN, bool STMA>
__global__ void __launch_bounds__(Cfg<BITS, MODE, BN>::THREADS, 1)
glu_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
              const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS0,
              const __grid_constant__ CUtensorMap tmQ0, const __grid_constant__ CUtensorMap tmS1,
              const __grid_constant__ CUtensorMap tmQ1, const Args args) {
  using C = Cfg<BITS, MODE, BN>;
  constexpr bool DUAL = C::DUAL;
  constexpr int RO1 = MODE == 2 ? BM : 0;  // row offset of the second matrix
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array, so that
  // every derived pointer stays a shared-memory pointer (ld/st.shared rather
  // than generic accesses)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sP = smem + C::OFF_P;
  int* plan = reinterpret_cast<int*>(smem + C::OFF_PLAN);
  int* s_goff = reinterpret_cast<int*>(smem + C::OFF_TILE);
  int* s_slot = s_goff + PLAN_MAX_GROUPS + 1;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* a_full = bars;                   // [SA] A stage ready (TMA tx or 8 dequant warps)
  uint64_t* a_empty = a_full + C::SA;        // [SA] A stage consumed (MMA commit)
  uint64_t* b_full = a_empty + C::SA;        // [SB] B stage landed (TMA tx)
  uint64_t* b_empty = b_full + C::SB;        // [SB] B stage consumed (MMA commit)
  uint64_t* p_full = b_empty + C::SB;        // [SP] packed stage landed (TMA tx)
  uint64_t* p_empty = p_full + C::SP;        // [SP] packed stage consumed (8 dequant warps)
  uint64_t* acc_full = p_empty + C::SP;      // [NACC] accumulator ready (MMA commit)
  uint64_t* acc_empty = acc_full + C::NACC;  // [NACC] accumulator drained (4 epilogue warps)
  uint64_t* s_full = acc_empty + C::NACC;    // [SS] scale chunk landed (TMA tx)
  uint64_t* s_empty = s_full + C::SS;        // [SS] scale chunk consumed (dequantiser warps)
  const uint8_t* sS = smem + C::OFF_S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Ctl ctl{abort_flag};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = args.K;
  const int NKB = K / BK;
  const int MT = args.OUT / C::ROWS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::SA; ++i) {
      mbar_init(&a_full[i], BITS == 16 ? 1 : C::DQW);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < C::SB; ++i) {
      mbar_init(&b_full[i], args.in_by_pos ? 1 : 32);  // TMA tx, or one cp.async arrival per producer lane
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < C::SP; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], C::DQW);
    }
    for (int i = 0; i < C::NACC; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    for (int i = 0; i < C::SS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], C::DQW);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // tile plan: plan[u] = first flat n-tile of group u (prefix of ceil(count / BN))
  const int U = args.dense_rows > 0 ? 1 : min(args.counts[0], args.max_groups);
  const bool tab_smem = C::TILE_SMEM && args.dense_rows == 0;
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int g0 = args.dense_rows > 0 ? 0 : args.group_off[u], g1 = args.dense_rows > 0 ? 0 : args.group_off[u + 1];
    const int cnt = args.dense_rows > 0 ? args.dense_rows : g1 - g0;
    plan[u + 1] = (cnt + BN - 1) / BN;
    if (tab_smem) {
      s_goff[u] = g0;
      s_slot[u] = args.slot_ids[u];
      if (u == U - 1) s_goff[U] = g1;
    }
  }
  const int* gtab = tab_smem ? s_goff : args.group_off;
  const int* stab = tab_smem ? s_slot : args.slot_ids;
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
    // ---------------------------------------------------------------- weight producer
    if (lane == 0) {
      int s_i = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      constexpr int RING = BITS == 16 ? C::SA : C::SP;
      uint64_t* full = BITS == 16 ? a_full : p_full;
      uint64_t* empty = BITS == 16 ? a_empty : p_empty;
      // scale/bias rows of a tile (contiguous, 128 rows x K/64 groups) go to
      // L2 one tile ahead, so the dequantisers' loads of them hit L2
      auto prefetch_scales = [&](int tt) {
        if (BITS == 16 || STMA || tt >= total) return;
        const Tile tn = tile_of<BN>(tt, plan, U, NT, args, gtab, stab);
        if (tn.slot < 0 || tn.slot >= args.num_slots) return;
        const int groups = K / 64;
        const size_t off = ((size_t)tn.slot * args.OUT + (size_t)tn.m * C::ROWS) * groups;
        const size_t off1 = off + (size_t)RO1 * groups;
        const uint32_t bytes = BM * groups * 2;
        prefetch_l2(args.s0 + off, bytes);
        prefetch_l2(args.b0 + off, bytes);
        if (DUAL) {
          prefetch_l2(args.s1 + off1, bytes);
          prefetch_l2(args.b1 + off1, bytes);
        }
      };
      prefetch_scales(blockIdx.x);
      int ss = 0, s_issued = 0;  // scale chunk ring (TMA-staged scales)
      uint32_t sph = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
        prefetch_scales(t + gridDim.x);
        const int row0 = tl.slot * args.OUT + tl.m * C::ROWS;
        const int nstage = BITS == 16 ? NKB : (NKB + C::KP - 1) / C::KP;
        for (int kb = 0; kb < nstage; ++kb) {
          if (STMA && (kb * C::KP) % 8 == 0) {
            // scales and biases of groups [kb*KP, kb*KP + 8) for the tile's
            // rows, ahead of the packed stages that use them
            ok = wait_bar(&s_empty[ss], sph ^ 1, ctl, BACKOFF_NS);
            if (!ok) break;
            uint8_t* dst = const_cast<uint8_t*>(sS) + ss * C::S_BYTES;
            mbar_expect_tx(&s_full[ss], C::S_BYTES);
            tma_load_2d(dst, &tmS0, kb * C::KP, row0, &s_full[ss]);
            tma_load_2d(dst + BM * 16, &tmQ0, kb * C::KP, row0, &s_full[ss]);
            if (DUAL) {
              tma_load_2d(dst + 2 * BM * 16, &tmS1, kb * C::KP, row0 + RO1, &s_full[ss]);
              tma_load_2d(dst + 3 * BM * 16, &tmQ1, kb * C::KP, row0 + RO1, &s_full[ss]);
            }
            ++s_issued;
            if (++ss == C::SS) { ss = 0; sph ^= 1; }
          }
          ok = wait_bar(&empty[s_i], ph ^ 1, ctl, BACKOFF_NS);
          if (!ok) break;
          if (BITS == 16) {
            mbar_expect_tx(&full[s_i], C::A_BYTES);
            tma_load_2d(sA + s_i * C::A_BYTES, &tmA0, kb * BK, row0, &full[s_i]);
            if (DUAL) tma_load_2d(sA + s_i * C::A_BYTES + C::A_MAT, &tmA1, kb * BK, row0 + RO1, &full[s_i]);
          } else {
            // 128 bytes of every row: columns beyond the row end are the TMA's
            // zero fill and are never dequantised
            mbar_expect_tx(&full[s_i], C::P_BYTES);
            const int col = kb * 32;  // packed uint32 column (32 words = 128 bytes)
            tma_load_2d(sP + s_i * C::P_BYTES, &tmA0, col, row0, &full[s_i]);
            if (DUAL) tma_load_2d(sP + s_i * C::P_BYTES + C::P_MAT, &tmA1, col, row0 + RO1, &full[s_i]);
          }
          ++issued;
          if (++s_i == RING) { s_i = 0; ph ^= 1; }
        }
      }
      if (!ok) {  // drain this thread's copies still in flight (bounded)
        for (int i = 0; i < min(issued, RING); ++i) {
          int s = s_i - 1 - i;
          uint32_t p = ph;
          if (s < 0) { s += RING; p ^= 1; }
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], p) && clock64() - t0 < WAIT_CYCLES) {
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
  } else if (warp == 2) {
    // ---------------------------------------------------------------- B row producer
    if (args.in_by_pos) {
      // B rows in dispatch order (dense mode, or rows permuted beforehand):
      // a tile's rows are contiguous, one TMA box (BN rows x 128 bytes, SW128,
      // zero fill past the last row) per operand stage; rows past the group's
      // pairs are read but their results are never written
      if (lane == 0) {
        int sb = 0, issued = 0;
        uint32_t pb = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
          const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
          for (int kb0 = 0; kb0 < NKB; kb0 += C::KBB) {
            ok = wait_bar(&b_empty[sb], pb ^ 1, ctl, BACKOFF_NS);
            if (!ok) break;
            const int nsub = min(C::KBB, NKB - kb0);
            mbar_expect_tx(&b_full[sb], nsub * C::B_SUB);
            for (int j = 0; j < nsub; ++j)
              tma_load_2d(sB + sb * C::B_BYTES + j * C::B_SUB, &tmB, (kb0 + j) * BK, tl.goff + tl.n0, &b_full[sb]);
            ++issued;
            if (++sb == C::SB) { sb = 0; pb ^= 1; }
          }
        }
        if (!ok) {  // drain the loads still in flight (bounded)
          for (int i = 0; i < min(issued, C::SB); ++i) {
            int st = sb - 1 - i;
            uint32_t p = pb;
            if (st < 0) { st += C::SB; p ^= 1; }
            const long long t0 = clock64();
            while (!mbar_try_wait(&b_full[st], p) && clock64() - t0 < WAIT_CYCLES) {
            }
          }
        }
      }
    } else {
    // Gathered rows: 16-byte LSU copies straight into the SW128 operand layout
    // (row j of a stage at 128 j, chunk c at c ^ (j & 7)); lane l copies chunk
    // l % 8 of rows l / 8 + 4 i.  Each lane reports its copies to the stage's
    // full barrier (32 arrivals); rows past the tile's pairs are zero.
    constexpr int RPL = BN / 4;  // rows per lane
    const int c = lane & 7, r0 = lane >> 3;
    const size_t row_bytes = static_cast<size_t>(K) * 2;
    int sb = 0;
    uint32_t pb = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
      int row[RPL];  // source row of each of this lane's tile rows, -1: zero fill
#pragma unroll
      for (int i = 0; i < RPL; ++i) {
        const int j = r0 + 4 * i;
        int rw = -1;
        if (j < tl.nvalid) {
          const int pos = tl.goff + tl.n0 + j;
          rw = args.in_by_pos ? pos : args.perm[pos] / args.pair_div;
        }
        row[i] = (rw >= 0 && rw < args.in_rows) ? rw : -1;
      }
      for (int kb0 = 0; kb0 < NKB; kb0 += C::KBB) {
        ok = wait_bar(&b_empty[sb], pb ^ 1, ctl, BACKOFF_NS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const int nsub = min(C::KBB, NKB - kb0);
        for (int j = 0; j < nsub; ++j) {
          uint8_t* dst = sB + sb * C::B_BYTES + j * C::B_SUB;
          const uint8_t* col = args.in + (kb0 + j) * (BK * 2) + c * 16;
#pragma unroll
          for (int i = 0; i < RPL; ++i) {
            const int rt = r0 + 4 * i;  // row within the tile
            const bool v = row[i] >= 0;
            cp_async16(dst + rt * 128 + ((c ^ (rt & 7)) << 4), v ? col + row[i] * row_bytes : args.in, v ? 16u : 0u);
          }
        }
        cp_async_arrive(&b_full[sb]);
        if (++sb == C::SB) { sb = 0; pb ^= 1; }
      }
    }
    cp_async_wait_all();  // no copy of this warp outlives the kernel
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16<BN>();
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        const int ab = it % C::NACC;
        const uint32_t accp = static_cast<uint32_t>((it / C::NACC) & 1);
        ok = wait_bar(&acc_empty[ab], accp ^ 1, ctl);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d0 = tmem + ab * C::ACC_COLS;
        for (int kb = 0; kb < NKB; ++kb) {
          const int jb = kb % C::KBB;  // operand stage within the B stage
          if (jb == 0) ok = wait_bar(&b_full[sb], pb, ctl);
          if (kb % C::MG == 0 && ok) {
            // dequantised stages fill in order (every dequantiser arrives on
            // them in turn), so the last stage of a group being full implies
            // the rest are: one wait per MG stages
            int sl = sa + min(C::MG, NKB - kb) - 1;
            uint32_t ph = pa;
            if (sl >= C::SA) { sl -= C::SA; ph ^= 1; }
            ok = wait_bar(&a_full[sl], ph, ctl);
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t b_base = smem_u32(sB + sb * C::B_BYTES + jb * C::B_SUB);
          if (C::ATM) {
            const uint32_t a_t = tmem + C::ACC_TOTAL + sa * C::NMAT * (BK / 2);
            const uint64_t bd0 = desc_sw128(b_base);  // +2 per 32-byte K step (address field is addr >> 4)
            umma_bf16_ts(d0, a_t, bd0, idesc, kb != 0);
            if (DUAL) umma_bf16_ts(d0 + BN, a_t + BK / 2, bd0, idesc, kb != 0);
#pragma unroll
            for (int kk = 1; kk < BK / 16; ++kk) {
              umma_bf16_ts(d0, a_t + kk * 8, bd0 + 2 * kk, idesc, 1u);
              if (DUAL) umma_bf16_ts(d0 + BN, a_t + BK / 2 + kk * 8, bd0 + 2 * kk, idesc, 1u);
            }
          } else {
            const uint32_t a_base = smem_u32(sA + sa * C::A_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t bd = desc_sw128(b_base + kk * 32);
              const uint32_t acc = (kb | kk) != 0;
              umma_bf16(d0, desc_sw128(a_base + kk * 32), bd, idesc, acc);
              if (DUAL) umma_bf16(d0 + BN, desc_sw128(a_base + C::A_MAT + kk * 32), bd, idesc, acc);
            }
          }
          umma_commit(&a_empty[sa]);
          if (++sa == C::SA) { sa = 0; pa ^= 1; }
          if (jb == C::KBB - 1 || kb == NKB - 1) {
            umma_commit(&b_empty[sb]);
            if (++sb == C::SB) { sb = 0; pb ^= 1; }
          }
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
    }
  } else if (warp >= DQ_WARP0 && warp < C::EPI_WARP0) {
    // ---------------------------------------------------------------- dequantisers
    if (BITS != 16) {
      if constexpr (STMA)
        dequant_role<BITS, MODE, BN, 1, true>(args, plan, U, NT, total, sA, sP, a_full, a_empty, p_full, p_empty,
                                              ctl, tmem, gtab, stab, sS, s_full, s_empty);
      else if ((K / 64) % 4 == 0)
        dequant_role<BITS, MODE, BN, 4, false>(args, plan, U, NT, total, sA, sP, a_full, a_empty, p_full, p_empty,
                                               ctl, tmem, gtab, stab, sS, s_full, s_empty);
      else
        dequant_role<BITS, MODE, BN, 1, false>(args, plan, U, NT, total, sA, sP, a_full, a_empty, p_full, p_empty,
                                               ctl, tmem, gtab, stab, sS, s_full, s_empty);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (last 4 warps)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const int ab = it % C::NACC;
      const uint32_t accp = static_cast<uint32_t>((it / C::NACC) & 1);
      const Tile tl = tile_of<BN>(t, plan, U, NT, args, gtab, stab);
      ok = wait_bar(&acc_full[ab], accp, ctl, BACKOFF_NS);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-wide
      if (!ok) break;
      tc_fence_after();
      const bool slot_ok = tl.slot >= 0 && tl.slot < args.num_slots;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + ab * C::ACC_COLS;
      const int ocol = tl.m * C::ROWS + r;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 32) {
        // output rows of pairs j0 .. j0+31, one per lane, broadcast by shuffle
        const int jl = j0 + lane;
        int my_row = 0;
        if (jl < tl.nvalid) {
          const int pos = tl.goff + tl.n0 + jl;
          my_row = args.out_by_pos ? pos : args.perm[pos];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int jb = j0 + 16 * h;
          if (jb >= BN) break;
          uint32_t g[16], u[16];
          tmem_ld16(tbase + jb, g);
          if (DUAL) tmem_ld16(tbase + BN + jb, u);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int orow = __shfl_sync(0xffffffffu, my_row, 16 * h + jj);
            if (jb + jj < tl.nvalid) {
              uint16_t v;
              if (!slot_ok) v = 0;
              else if (MODE == 1) v = swiglu_bf16(__uint_as_float(g[jj]), __uint_as_float(u[jj]));
              else v = f32_to_bf16(__uint_as_float(g[jj]));
              args.out[(size_t)orow * args.OUT + ocol] = v;
              if (MODE == 2)  // the second 128-row half of the tile
                args.out[(size_t)orow * args.OUT + ocol + BM] = slot_ok ? f32_to_bf16(__uint_as_float(u[jj])) : 0;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
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
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                     uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * esize};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BITS, int MODE, int BN>
static int launch_cfg(const sg_arena* A, const Args& args_in, cudaStream_t s) {
  using C = Cfg<BITS, MODE, BN>;
  constexpr bool DUAL = C::DUAL;
  Args args = args_in;
  const int K = args.K, OUT = args.OUT;
  const uint64_t rows_total = (uint64_t)A->num_slots * OUT;
  CUtensorMap m0, m1, mb, ms0, mq0, ms1, mq1;
  const void* w0 = MODE == 1 ? A->gate_w : A->down_w;
  const void* w1 = MODE == 1 ? A->up_w : A->down_w;
  bool ok;
  if (BITS == 16) {
    ok = make_map(&m0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w0, K, rows_total, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map(&m1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w1, K, rows_total, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t words = (uint64_t)K * BITS / 32;
    ok = make_map(&m0, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w0, words, rows_total, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w1, words, rows_total, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  // B rows in dispatch order: [in_rows, K] bf16, box BN rows x 64 columns
  if (args.in_by_pos)
    ok = ok && make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.in, K, (uint64_t)args.in_rows, BK, BN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  else
    memset(&mb, 0, sizeof(mb));
  // scale/bias chunks by TMA: [rows_total, K/64] bf16, box 8 groups x 128 rows
  // (needs 16-byte row strides: group counts that are multiples of 8)
  const int groups = K / 64;
  const bool scale_tma = C::SS > 0 && groups % 8 == 0;
  memset(&ms0, 0, sizeof(ms0));
  memset(&mq0, 0, sizeof(mq0));
  memset(&ms1, 0, sizeof(ms1));
  memset(&mq1, 0, sizeof(mq1));
  if (scale_tma)
    ok = ok &&
         make_map(&ms0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.s0, groups, rows_total, 8, BM,
                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
         make_map(&mq0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.b0, groups, rows_total, 8, BM,
                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
         make_map(&ms1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.s1, groups, rows_total, 8, BM,
                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
         make_map(&mq1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.b1, groups, rows_total, 8, BM,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return SG_ERR_CUDA;
  static bool attr_done[64] = {};  // per device
  int dev = 0;
  SG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
  if (!attr_done[dev]) {
    SG_CUDA_TRY(cudaFuncSetAttribute(glu_tc_kernel<BITS, MODE, BN, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    if constexpr (C::SS > 0)
      SG_CUDA_TRY(cudaFuncSetAttribute(glu_tc_kernel<BITS, MODE, BN, true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_done[dev] = true;
  }
  int grid = num_sms();
  if (args.dense_rows > 0) {  // the tile count is known on the host: no idle CTAs
    const int tiles = (args.OUT / C::ROWS) * ((args.dense_rows + BN - 1) / BN);
    grid = tiles < grid ? tiles : grid;
  }
  if constexpr (C::SS > 0) {
    if (scale_tma) {
      glu_tc_kernel<BITS, MODE, BN, true><<<grid, C::THREADS, C::SMEM, s>>>(m0, m1, mb, ms0, mq0, ms1, mq1, args);
      SG_LAUNCH_CHECK();
      return SG_OK;
    }
  }
  glu_tc_kernel<BITS, MODE, BN, false><<<grid, C::THREADS, C::SMEM, s>>>(m0, m1, mb, ms0, mq0, ms1, mq1, args);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

template <int BITS, int MODE>
static int launch_bits(const sg_arena* A, int bn, const Args& args, cudaStream_t s) {
  switch (bn) {
    case 16: return launch_cfg<BITS, MODE, 16>(A, args, s);
    case 32: return launch_cfg<BITS, MODE, 32>(A, args, s);
    case 64: return launch_cfg<BITS, MODE, 64>(A, args, s);
    default: return launch_cfg<BITS, MODE, 128>(A, args, s);
  }
}

// gate/up: mode 1; down: 256-row paired tiles (mode 2) when the output
// dimension allows, else 128-row tiles (mode 0)
static int mode_of(bool dual, int OUT) { return dual ? 1 : (OUT % (2 * BM) == 0 ? 2 : 0); }

template <int BITS>
static int launch_mode(const sg_arena* A, int mode, int bn, const Args& args, cudaStream_t s) {
  switch (mode) {
    case 1: return launch_bits<BITS, 1>(A, bn, args, s);
    case 2: return launch_bits<BITS, 2>(A, bn, args, s);
    default: return launch_bits<BITS, 0>(A, bn, args, s);
  }
}

}  // namespace tc

// Choose BN from the mean pairs per group (host-side bound: P / grid_groups),
// unless sg_set_glu_tile fixed one.
static int g_tc_tile = 0;
static int pick_bn(int P, int grid_groups) {
  if (g_tc_tile) return g_tc_tile;
  const int avg = (P + grid_groups - 1) / (grid_groups > 0 ? grid_groups : 1);
  if (avg <= 16) return 16;
  if (avg <= 32) return 32;
  if (avg <= 64) return 64;
  return 128;
}

bool tc_supported(const sg_arena* A, bool dual, int grid_groups) {
  const int K = dual ? A->hidden : A->inter;
  const int OUT = dual ? A->inter : A->hidden;
  // packed rows must fill one 128-byte TMA box
  return K % tc::BK == 0 && OUT % tc::BM == 0 && grid_groups <= tc::PLAN_MAX_GROUPS &&
         (A->bits == 16 || K * A->bits / 8 >= 128);
}

int tc_glu_launch(const sg_arena* A, bool dual, const uint16_t* in, int in_rows, int pair_div, int in_by_pos,
                  int out_by_pos, int P, const int32_t* counts, const int32_t* slot_ids, const int32_t* group_off,
                  const int32_t* perm, int grid_groups, uint16_t* out, cudaStream_t s) {
  tc::Args a;
  a.num_slots = A->num_slots;
  a.K = dual ? A->hidden : A->inter;
  a.OUT = dual ? A->inter : A->hidden;
  a.s0 = static_cast<const uint16_t*>(dual ? A->gate_s : A->down_s);
  a.b0 = static_cast<const uint16_t*>(dual ? A->gate_b : A->down_b);
  a.s1 = static_cast<const uint16_t*>(dual ? A->up_s : A->down_s);
  a.b1 = static_cast<const uint16_t*>(dual ? A->up_b : A->down_b);
  a.in = reinterpret_cast<const uint8_t*>(in);
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
  a.dense_rows = 0;
  a.dense_slot = 0;
  const int bn = pick_bn(P, grid_groups);
  switch (A->bits) {
    case 16: return tc::launch_mode<16>(A, tc::mode_of(dual, a.OUT), bn, a, s);
    case 8: return tc::launch_mode<8>(A, tc::mode_of(dual, a.OUT), bn, a, s);
    default: return tc::launch_mode<4>(A, tc::mode_of(dual, a.OUT), bn, a, s);
  }
}

// Dense mode: all `rows` rows of `in` through slot `sid` (the shared expert).
// Pair tiles of 64 keep the tensor-memory operand path while the tiles fit in
// one wave of CTAs; wider problems take 128-wide tiles (less re-dequantisation).
int tc_dense_launch(const sg_arena* A, bool dual, const uint16_t* in, int rows, int sid, uint16_t* out,
                    cudaStream_t s) {
  tc::Args a;
  memset(&a, 0, sizeof(a));
  a.num_slots = A->num_slots;
  a.K = dual ? A->hidden : A->inter;
  a.OUT = dual ? A->inter : A->hidden;
  a.s0 = static_cast<const uint16_t*>(dual ? A->gate_s : A->down_s);
  a.b0 = static_cast<const uint16_t*>(dual ? A->gate_b : A->down_b);
  a.s1 = static_cast<const uint16_t*>(dual ? A->up_s : A->down_s);
  a.b1 = static_cast<const uint16_t*>(dual ? A->up_b : A->down_b);
  a.in = reinterpret_cast<const uint8_t*>(in);
  a.in_rows = rows;
  a.pair_div = 1;
  a.in_by_pos = 1;
  a.out_by_pos = 1;
  a.max_groups = 1;
  a.out = out;
  a.dense_rows = rows;
  a.dense_slot = sid;
  const int mt = a.OUT / (tc::mode_of(dual, a.OUT) == 2 ? 2 * tc::BM : tc::BM);
  int bn = rows > 32 ? 64 : (rows > 16 ? 32 : 16);
  if ((long long)mt * ((rows + 63) / 64) > tc::num_sms()) bn = 128;
  switch (A->bits) {
    case 16: return tc::launch_mode<16>(A, tc::mode_of(dual, a.OUT), bn, a, s);
    case 8: return tc::launch_mode<8>(A, tc::mode_of(dual, a.OUT), bn, a, s);
    default: return tc::launch_mode<4>(A, tc::mode_of(dual, a.OUT), bn, a, s);
  }
}

}  // namespace sg

// the integer-operand gate/up kernel shares this unit's helpers and status word
#include "sg_glu_i8.cuh"

namespace sg {
int ep_device_status(int reset);  // the expert-parallel exchange kernels' word (sg_ep.cu)
}

extern "C" int sg_device_status(int reset) {
  int v = 0;
  SG_CUDA_TRY(cudaMemcpyFromSymbol(&v, sg::g_device_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SG_CUDA_TRY(cudaMemcpyToSymbol(sg::g_device_status, &zero, sizeof(int)));
  }
  const int ep = sg::ep_device_status(reset);
  return v ? v : ep;
}
