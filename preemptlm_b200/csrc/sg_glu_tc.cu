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
// Warp roles (11 warps, one CTA per SM, persistent over a static tile list):
//   w0      TMA producer of weight tiles: bf16 straight into the SW128 operand
//           layout, or packed 8/4-bit words (SW64 / SW32) for the dequantisers
//   w1      TMEM allocation + single-thread tcgen05.mma issue + commits
//   w2      TMA gather4 producer of the B rows (token rows picked by the
//           dispatch permutation)
//   w3-w6   dequantisers (quantised arenas): thread r owns row r of the tile,
//           w = bf16(scale * q + bias) written in the SW128 operand layout
//   w7-w10  epilogue: tcgen05.ld -> SwiGLU / bf16 -> global, one warp per
//           32-lane TMEM quadrant
//
// Every mbarrier wait is bounded (about one second of clock64); on expiry the
// CTA records SG_ERR_TIMEOUT in the library's device status word, drains the
// copies it issued (bounded as well), frees its TMEM and returns.
#include <cuda.h>

#include <mutex>

#include "sg_common.cuh"

namespace sg {

__device__ int g_device_status = 0;  // first error recorded by a kernel of this library

namespace tc {

constexpr int BM = 128;            // weight rows per tile (MMA M)
constexpr int BK = 64;             // K per pipeline stage (one 128-byte swizzle atom of bf16)
constexpr int NUM_WARPS = 11;
constexpr int NUM_THREADS = NUM_WARPS * 32;
constexpr int RING_BUDGET = 192 * 1024;
constexpr int PLAN_MAX_GROUPS = 2048;
constexpr long long WAIT_CYCLES = 2000000000LL;  // ~1 s

__host__ __device__ constexpr int pow2ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }

template <int BITS, bool DUAL, int BN>
struct Cfg {
  static constexpr int NMAT = DUAL ? 2 : 1;
  static constexpr int A_MAT = BM * BK * 2;                       // one bf16 operand tile
  static constexpr int A_BYTES = NMAT * A_MAT;
  static constexpr int P_MAT = BITS == 16 ? 0 : BM * BK * BITS / 8;  // one packed tile
  static constexpr int P_BYTES = NMAT * P_MAT;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int SA = BITS == 16 ? cmin(8, RING_BUDGET / (A_BYTES + B_BYTES)) : (DUAL ? 3 : 4);
  static constexpr int SP = BITS == 16 ? 0 : cmin(8, (RING_BUDGET - SA * (A_BYTES + B_BYTES)) / P_BYTES);
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int NACC = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = pow2ceil(NACC * ACC_COLS < 32 ? 32 : NACC * ACC_COLS);
  // shared memory carve-up (offsets from a 1024-aligned base)
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + SA * A_BYTES;
  static constexpr int OFF_P = OFF_B + SA * B_BYTES;
  static constexpr int OFF_PLAN = OFF_P + SP * P_BYTES;
  static constexpr int OFF_ROWS = (OFF_PLAN + (PLAN_MAX_GROUPS + 1) * 4 + 15) & ~15;
  static constexpr int OFF_BAR = (OFF_ROWS + BN * 4 + 15) & ~15;
  static constexpr int NUM_BARS = 3 * SA + 2 * SP + 2 * NACC;
  static constexpr int SMEM = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + tmem slot/abort flag + align slack
  static_assert(SA >= 2 && (BITS == 16 || SP >= 2), "pipeline too shallow");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(B_BYTES % 1024 == 0, "B tile must keep 1024-byte alignment");
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

struct Ctl {
  volatile int* abort;  // shared flag: a wait in this CTA expired
};

// Bounded wait for the phase of parity `parity` to complete.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctl ctl) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
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
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int col, int r0, int r1, int r2, int r3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
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
__device__ __forceinline__ float qf(uint32_t q) {  // exact small unsigned int -> fp32
  return __fsub_rn(__uint_as_float(0x4B000000u | q), 8388608.0f);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Row r of one packed stage tile -> 64 bf16 (8 x 16-byte chunks) in the SW128
// operand layout of the A stage tile.
template <int BITS>
__device__ __forceinline__ void dequant_row(const uint8_t* p_tile, uint8_t* a_tile, int r, float s, float b) {
  uint8_t* arow = a_tile + r * 128;
  if (BITS == 8) {
    // SW64 packed tile: 64-byte rows, 16-byte chunk c at c ^ ((r >> 1) & 3)
    const uint8_t* prow = p_tile + r * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(prow + ((c ^ ((r >> 1) & 3)) << 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // output chunk oc = 2c + h holds weights 8oc .. 8oc+7
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t word = w[2 * h + (q >> 1)];
          const int sh = (q & 1) * 16;
          op[q] = pack_bf16x2(fmaf(qf((word >> sh) & 0xFFu), s, b), fmaf(qf((word >> (sh + 8)) & 0xFFu), s, b));
        }
        const int oc = 2 * c + h;
        *reinterpret_cast<uint4*>(arow + ((oc ^ (r & 7)) << 4)) = o;
      }
    }
  } else {
    // SW32 packed tile: 32-byte rows, 16-byte chunk c at c ^ ((r >> 2) & 1)
    const uint8_t* prow = p_tile + r * 32;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(prow + ((c ^ ((r >> 2) & 1)) << 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {  // output chunk oc = 4c + h = one 32-bit word (8 weights)
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
        const uint32_t word = w[h];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          op[q] = pack_bf16x2(fmaf(qf((word >> (8 * q)) & 0xFu), s, b), fmaf(qf((word >> (8 * q + 4)) & 0xFu), s, b));
        const int oc = 4 * c + h;
        *reinterpret_cast<uint4*>(arow + ((oc ^ (r & 7)) << 4)) = o;
      }
    }
  }
}

// ------------------------------------------------------------------ arguments
struct Args {
  int num_slots, K, OUT;
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
};

struct Tile {
  int u, m, n0, nvalid, slot, goff;
};

template <int BN>
__device__ __forceinline__ Tile tile_of(int t, const int* plan, int U, int NT, const Args& a) {
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
  tl.goff = a.group_off[lo];
  const int cnt = a.group_off[lo + 1] - tl.goff;
  tl.nvalid = min(BN, cnt - tl.n0);
  tl.slot = a.slot_ids[lo];
  return tl;
}

// ------------------------------------------------------------------ the kernel
template <int BITS, bool DUAL, int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
glu_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
              const __grid_constant__ CUtensorMap tmB, const Args args) {
  using C = Cfg<BITS, DUAL, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sP = smem + C::OFF_P;
  int* plan = reinterpret_cast<int*>(smem + C::OFF_PLAN);
  int* rows = reinterpret_cast<int*>(smem + C::OFF_ROWS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* a_full = bars;                   // [SA] A stage ready (TMA tx or 4 dequant warps)
  uint64_t* b_full = a_full + C::SA;         // [SA] B stage ready (TMA tx)
  uint64_t* a_empty = b_full + C::SA;        // [SA] A+B stage consumed (MMA commit)
  uint64_t* p_full = a_empty + C::SA;        // [SP] packed stage landed (TMA tx)
  uint64_t* p_empty = p_full + C::SP;        // [SP] packed stage consumed (4 dequant warps)
  uint64_t* acc_full = p_empty + C::SP;      // [NACC] accumulator ready (MMA commit)
  uint64_t* acc_empty = acc_full + C::NACC;  // [NACC] accumulator drained (4 epilogue warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Ctl ctl{abort_flag};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = args.K;
  const int NKB = K / BK;
  const int MT = args.OUT / BM;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::SA; ++i) {
      mbar_init(&a_full[i], BITS == 16 ? 1 : 4);
      mbar_init(&b_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < C::SP; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], 4);
    }
    for (int i = 0; i < C::NACC; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // tile plan: plan[u] = first flat n-tile of group u (prefix of ceil(count / BN))
  const int U = min(args.counts[0], args.max_groups);
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int cnt = args.group_off[u + 1] - args.group_off[u];
    plan[u + 1] = (cnt + BN - 1) / BN;
  }
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
      int sa = 0, sp = 0;
      uint32_t pa = 0, pp = 0;  // phase bits
      int issued_a = 0, issued_p = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = tile_of<BN>(t, plan, U, NT, args);
        const int row0 = tl.slot * args.OUT + tl.m * BM;
        for (int kb = 0; kb < NKB && ok; ++kb) {
          if (BITS == 16) {
            ok = wait_bar(&a_empty[sa], pa ^ 1, ctl);
            if (!ok) break;
            mbar_expect_tx(&a_full[sa], C::A_BYTES);
            tma_load_2d(sA + sa * C::A_BYTES, &tmA0, kb * BK, row0, &a_full[sa]);
            if (DUAL) tma_load_2d(sA + sa * C::A_BYTES + C::A_MAT, &tmA1, kb * BK, row0, &a_full[sa]);
            ++issued_a;
            if (++sa == C::SA) { sa = 0; pa ^= 1; }
          } else {
            ok = wait_bar(&p_empty[sp], pp ^ 1, ctl);
            if (!ok) break;
            mbar_expect_tx(&p_full[sp], C::P_BYTES);
            const int col = kb * BK * BITS / 32;  // packed uint32 column
            tma_load_2d(sP + sp * C::P_BYTES, &tmA0, col, row0, &p_full[sp]);
            if (DUAL) tma_load_2d(sP + sp * C::P_BYTES + C::P_MAT, &tmA1, col, row0, &p_full[sp]);
            ++issued_p;
            if (++sp == C::SP) { sp = 0; pp ^= 1; }
          }
        }
      }
      if (!ok) {  // drain this thread's copies still in flight (bounded)
        Ctl drain_ctl = ctl;
        int depth = BITS == 16 ? min(issued_a, C::SA) : min(issued_p, C::SP);
        for (int i = 0; i < depth; ++i) {
          int s = (BITS == 16 ? sa : sp) - 1 - i;
          uint32_t ph = BITS == 16 ? pa : pp;
          const int ring = BITS == 16 ? C::SA : C::SP;
          if (s < 0) { s += ring; ph ^= 1; }
          uint64_t* fb = BITS == 16 ? &a_full[s] : &p_full[s];
          const long long t0 = clock64();
          while (!mbar_try_wait(fb, ph) && clock64() - t0 < WAIT_CYCLES) {
          }
          (void)drain_ctl;
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- B gather producer
    int sa = 0;
    uint32_t pa = 0;
    bool ok = true;
    int issued = 0;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const Tile tl = tile_of<BN>(t, plan, U, NT, args);
      __syncwarp();
      for (int j = lane; j < BN; j += 32) {
        const int pos = tl.goff + tl.n0 + (j < tl.nvalid ? j : 0);
        rows[j] = args.in_by_pos ? pos : args.perm[pos] / args.pair_div;
      }
      __syncwarp();
      if (lane == 0) {
        for (int kb = 0; kb < NKB; ++kb) {
          ok = wait_bar(&a_empty[sa], pa ^ 1, ctl);
          if (!ok) break;
          mbar_expect_tx(&b_full[sa], C::B_BYTES);
          uint8_t* dst = sB + sa * C::B_BYTES;
#pragma unroll 1
          for (int g = 0; g < BN / 4; ++g)
            tma_gather4(dst + g * 512, &tmB, kb * BK, rows[4 * g], rows[4 * g + 1], rows[4 * g + 2],
                        rows[4 * g + 3], &b_full[sa]);
          ++issued;
          if (++sa == C::SA) { sa = 0; pa ^= 1; }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (!ok && lane == 0) {
      for (int i = 0; i < min(issued, C::SA); ++i) {
        int s = sa - 1 - i;
        uint32_t ph = pa;
        if (s < 0) { s += C::SA; ph ^= 1; }
        const long long t0 = clock64();
        while (!mbar_try_wait(&b_full[s], ph) && clock64() - t0 < WAIT_CYCLES) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16<BN>();
      int sa = 0;
      uint32_t pa = 0;
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
          ok = wait_bar(&a_full[sa], pa, ctl) && wait_bar(&b_full[sa], pa, ctl);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + sa * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + sa * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = desc_sw128(b_base + kk * 32);
            const uint32_t acc = (kb | kk) != 0;
            umma_bf16(d0, desc_sw128(a_base + kk * 32), bd, idesc, acc);
            if (DUAL) umma_bf16(d0 + BN, desc_sw128(a_base + C::A_MAT + kk * 32), bd, idesc, acc);
          }
          umma_commit(&a_empty[sa]);
          if (++sa == C::SA) { sa = 0; pa ^= 1; }
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
    }
  } else if (warp >= 3 && warp <= 6) {
    // ---------------------------------------------------------------- dequantisers
    if (BITS != 16) {
      const int r = (warp - 3) * 32 + lane;
      const int groups = K / 64;
      int sa = 0, sp = 0;
      uint32_t pa = 0, pp = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = tile_of<BN>(t, plan, U, NT, args);
        // a slot outside the arena (a miss) reads no scales: its A tile is the
        // TMA's zero fill, its outputs are written as zeros by the epilogue
        const bool sok = tl.slot >= 0 && tl.slot < args.num_slots;
        const size_t row = sok ? (size_t)tl.slot * args.OUT + tl.m * BM + r : 0;
        const uint16_t* s0 = args.s0 + row * groups;
        const uint16_t* b0 = args.b0 + row * groups;
        const uint16_t* s1 = DUAL ? args.s1 + row * groups : nullptr;
        const uint16_t* b1 = DUAL ? args.b1 + row * groups : nullptr;
        float ns0 = 0.f, nb0 = 0.f, ns1 = 0.f, nb1 = 0.f;
        if (sok) {
          ns0 = bf16_to_f32(s0[0]);
          nb0 = bf16_to_f32(b0[0]);
          if (DUAL) {
            ns1 = bf16_to_f32(s1[0]);
            nb1 = bf16_to_f32(b1[0]);
          }
        }
        for (int kb = 0; kb < NKB; ++kb) {
          const float cs0 = ns0, cb0 = nb0, cs1 = ns1, cb1 = nb1;
          if (sok && kb + 1 < NKB) {  // one group ahead
            ns0 = bf16_to_f32(s0[kb + 1]);
            nb0 = bf16_to_f32(b0[kb + 1]);
            if (DUAL) {
              ns1 = bf16_to_f32(s1[kb + 1]);
              nb1 = bf16_to_f32(b1[kb + 1]);
            }
          }
          ok = wait_bar(&p_full[sp], pp, ctl) && wait_bar(&a_empty[sa], pa ^ 1, ctl);
          ok = __all_sync(0xffffffffu, ok);  // keep the warp converged for __syncwarp
          if (!ok) break;
          const uint8_t* ptile = sP + sp * C::P_BYTES;
          uint8_t* atile = sA + sa * C::A_BYTES;
          dequant_row<BITS>(ptile, atile, r, cs0, cb0);
          if (DUAL) dequant_row<BITS>(ptile + C::P_MAT, atile + C::A_MAT, r, cs1, cb1);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&a_full[sa]);
            mbar_arrive(&p_empty[sp]);
          }
          if (++sa == C::SA) { sa = 0; pa ^= 1; }
          if (++sp == C::SP) { sp = 0; pp ^= 1; }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 7-10)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const int ab = it % C::NACC;
      const uint32_t accp = static_cast<uint32_t>((it / C::NACC) & 1);
      ok = wait_bar(&acc_full[ab], accp, ctl);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-wide
      if (!ok) break;
      tc_fence_after();
      const Tile tl = tile_of<BN>(t, plan, U, NT, args);
      const bool slot_ok = tl.slot >= 0 && tl.slot < args.num_slots;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + ab * C::ACC_COLS;
      const int ocol = tl.m * BM + r;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        uint32_t g[16], u[16];
        tmem_ld16(tbase + j0, g);
        if (DUAL) tmem_ld16(tbase + BN + j0, u);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = j0 + jj;
          if (j < tl.nvalid) {
            const int pos = tl.goff + tl.n0 + j;
            const int orow = args.out_by_pos ? pos : args.perm[pos];
            uint16_t v;
            if (!slot_ok) v = 0;
            else if (DUAL) v = swiglu_bf16(__uint_as_float(g[jj]), __uint_as_float(u[jj]));
            else v = f32_to_bf16(__uint_as_float(g[jj]));
            args.out[(size_t)orow * args.OUT + ocol] = v;
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

template <int BITS, bool DUAL, int BN>
static int launch_cfg(const sg_arena* A, const uint16_t* in, int in_rows, const Args& args, cudaStream_t s) {
  using C = Cfg<BITS, DUAL, BN>;
  const int K = args.K, OUT = args.OUT;
  const uint64_t rows_total = (uint64_t)A->num_slots * OUT;
  CUtensorMap m0, m1, mb;
  const void* w0 = DUAL ? A->gate_w : A->down_w;
  const void* w1 = DUAL ? A->up_w : A->down_w;
  bool ok;
  if (BITS == 16) {
    ok = make_map(&m0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w0, K, rows_total, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map(&m1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w1, K, rows_total, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t words = (uint64_t)K * BITS / 32;
    const uint32_t box = BK * BITS / 32;
    const CUtensorMapSwizzle sw = BITS == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
    ok = make_map(&m0, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w0, words, rows_total, box, BM, sw) &&
         make_map(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w1, words, rows_total, box, BM, sw);
  }
  ok = ok && make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, in, K, (uint64_t)in_rows, BK, 1,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) return SG_ERR_CUDA;
  static bool attr_done = false;
  if (!attr_done) {
    SG_CUDA_TRY(cudaFuncSetAttribute(glu_tc_kernel<BITS, DUAL, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM));
    attr_done = true;
  }
  glu_tc_kernel<BITS, DUAL, BN><<<num_sms(), NUM_THREADS, C::SMEM, s>>>(m0, m1, mb, args);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

template <int BITS, bool DUAL>
static int launch_bits(const sg_arena* A, const uint16_t* in, int in_rows, int bn, const Args& args,
                       cudaStream_t s) {
  switch (bn) {
    case 16: return launch_cfg<BITS, DUAL, 16>(A, in, in_rows, args, s);
    case 32: return launch_cfg<BITS, DUAL, 32>(A, in, in_rows, args, s);
    case 64: return launch_cfg<BITS, DUAL, 64>(A, in, in_rows, args, s);
    default: return launch_cfg<BITS, DUAL, 128>(A, in, in_rows, args, s);
  }
}

}  // namespace tc

// Choose BN from the mean pairs per group (host-side bound: P / grid_groups).
static int pick_bn(int P, int grid_groups) {
  const int avg = (P + grid_groups - 1) / (grid_groups > 0 ? grid_groups : 1);
  if (avg <= 16) return 16;
  if (avg <= 32) return 32;
  if (avg <= 64) return 64;
  return 128;
}

bool tc_supported(const sg_arena* A, bool dual, int grid_groups) {
  const int K = dual ? A->hidden : A->inter;
  const int OUT = dual ? A->inter : A->hidden;
  return K % tc::BK == 0 && OUT % tc::BM == 0 && grid_groups <= tc::PLAN_MAX_GROUPS;
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
  a.counts = counts;
  a.slot_ids = slot_ids;
  a.group_off = group_off;
  a.perm = perm;
  a.pair_div = pair_div;
  a.in_by_pos = in_by_pos;
  a.out_by_pos = out_by_pos;
  a.max_groups = grid_groups;
  a.out = out;
  const int bn = pick_bn(P, grid_groups);
  switch (A->bits) {
    case 16: return dual ? tc::launch_bits<16, true>(A, in, in_rows, bn, a, s) : tc::launch_bits<16, false>(A, in, in_rows, bn, a, s);
    case 8: return dual ? tc::launch_bits<8, true>(A, in, in_rows, bn, a, s) : tc::launch_bits<8, false>(A, in, in_rows, bn, a, s);
    default: return dual ? tc::launch_bits<4, true>(A, in, in_rows, bn, a, s) : tc::launch_bits<4, false>(A, in, in_rows, bn, a, s);
  }
}

}  // namespace sg

extern "C" int sg_device_status(int reset) {
  int v = 0;
  SG_CUDA_TRY(cudaMemcpyFromSymbol(&v, sg::g_device_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SG_CUDA_TRY(cudaMemcpyToSymbol(sg::g_device_status, &zero, sizeof(int)));
  }
  return v;
}
