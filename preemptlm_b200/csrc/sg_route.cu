// Router logits (a1), softmax/top-k/renorm (a2) and the device-side unique /
// inverse / slot lookup / pair permutation (a3, a6) of the slotted MoE block.
#include "sg_common.cuh"

namespace sg {

// ============================================================== router logits
// CTA = 8 warps; a CTA covers RT_TOK tokens x (8 * RT_EXP) experts.  Each warp
// owns RT_EXP experts and all RT_TOK tokens of the tile; lane j accumulates
// h = 256*i + 8*j + e in (i, e) order, then every (expert, token) partial is
// folded 16, 8, 4, 2, 1 across the warp.  Tokens go in pairs through packed
// fma.rn.f32x2 (two accumulators, one instruction; each lane's FMA rounds as
// a scalar FMA would, so the order and the bits are those of one accumulator
// per (expert, token)).  x for the token tile is staged in shared memory as
// bf16x2 words holding a token pair's element h, laid out so that a lane's
// four pairs for one h are one 16-byte load; router rows stream from global
// (read once per token tile).
constexpr int RT_TOK = 8;
constexpr int RT_EXP = 4;
constexpr int RT_WARPS = 8;
constexpr int RT_PAIRS = RT_TOK / 2;

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}

__global__ void __launch_bounds__(RT_WARPS * 32)
router_logits_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                     uint16_t* __restrict__ logits, int T, int H, int E) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // word ((i * 8 + e) * 32 + j) * 4 + p = (x[t0 + 2p][h], x[t0 + 2p + 1][h]), h = 256 i + 8 j + e
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * RT_TOK;
  const int e0 = (blockIdx.y * RT_WARPS + warp) * RT_EXP;
  const int chunks = H >> 3;  // 16-byte chunks per row

  for (int it = threadIdx.x; it < RT_PAIRS * chunks; it += blockDim.x) {
    const int p = it / chunks, c = it - p * chunks;
    const int ta = t0 + 2 * p, tb = ta + 1;
    const uint4 va = ta < T ? reinterpret_cast<const uint4*>(x + (size_t)ta * H)[c] : make_uint4(0, 0, 0, 0);
    const uint4 vb = tb < T ? reinterpret_cast<const uint4*>(x + (size_t)tb * H)[c] : make_uint4(0, 0, 0, 0);
    const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
    const int i = c >> 5, j = c & 31;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xs[((i * 8 + 2 * q) * 32 + j) * 4 + p] = __byte_perm(wa[q], wb[q], 0x5410);      // element 2q
      xs[((i * 8 + 2 * q + 1) * 32 + j) * 4 + p] = __byte_perm(wa[q], wb[q], 0x7632);  // element 2q + 1
    }
  }
  __syncthreads();

  unsigned long long acc[RT_EXP][RT_PAIRS];
#pragma unroll
  for (int a = 0; a < RT_EXP; ++a)
#pragma unroll
    for (int b = 0; b < RT_PAIRS; ++b) acc[a][b] = 0ull;

  const int iters = H >> 8;
  // router rows: this lane's 16-byte chunk of iteration i + 1 is in flight
  // while iteration i computes
  uint4 wn[RT_EXP];
#pragma unroll
  for (int a = 0; a < RT_EXP; ++a) {
    const int e = e0 + a;
    wn[a] = (e < E) ? ldg_nc_v4(w + (size_t)e * H + (size_t)lane * 8) : make_uint4(0, 0, 0, 0);
  }
  for (int i = 0; i < iters; ++i) {
    uint4 wv[RT_EXP];
#pragma unroll
    for (int a = 0; a < RT_EXP; ++a) {
      wv[a] = wn[a];
      const int e = e0 + a;
      if (i + 1 < iters && e < E) wn[a] = ldg_nc_v4(w + (size_t)e * H + (size_t)((i + 1) * 32 + lane) * 8);
    }
#pragma unroll
    for (int el = 0; el < 8; ++el) {  // element order within the lane's chunk
      const uint4 xv = *reinterpret_cast<const uint4*>(xs + ((i * 8 + el) * 32 + lane) * 4);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      unsigned long long xp[RT_PAIRS];
#pragma unroll
      for (int p = 0; p < RT_PAIRS; ++p) xp[p] = pack2(lo_bf16(xw[p]), hi_bf16(xw[p]));
#pragma unroll
      for (int a = 0; a < RT_EXP; ++a) {
        const uint32_t ww[4] = {wv[a].x, wv[a].y, wv[a].z, wv[a].w};
        const float wf = (el & 1) ? hi_bf16(ww[el >> 1]) : lo_bf16(ww[el >> 1]);
        const unsigned long long w2 = pack2(wf, wf);
#pragma unroll
        for (int p = 0; p < RT_PAIRS; ++p)
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[a][p]) : "l"(xp[p]), "l"(w2));
      }
    }
  }
#pragma unroll
  for (int a = 0; a < RT_EXP; ++a) {
#pragma unroll
    for (int b = 0; b < RT_TOK; ++b) {
      const unsigned long long pr = acc[a][b >> 1];
      const float v = __uint_as_float(static_cast<uint32_t>((b & 1) ? (pr >> 32) : pr));
      const float sum = warp_fold_sum(v);
      const int e = e0 + a, t = t0 + b;
      if (lane == ((a * RT_TOK + b) & 31) && e < E && t < T) logits[(size_t)t * E + e] = f32_to_bf16(sum);
    }
  }
}

// Few experts (the shared expert's one-row gate): one warp per (token, expert)
// with the same per-lane order and fold as the tiled kernel above, so the
// logits are bit-identical to it.
__global__ void __launch_bounds__(256)
router_logits_small_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                           uint16_t* __restrict__ logits, int T, int H, int E) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= T * E) return;
  const int t = gw / E, e = gw - t * E;
  const uint16_t* xr = x + (size_t)t * H;
  const uint16_t* wr = w + (size_t)e * H;
  float acc = 0.0f;
  for (int i = 0; i < (H >> 8); ++i) {
    const int cc = i * 32 + lane;
    const uint4 xv = ldg_nc_v4(xr + (size_t)cc * 8);
    const uint4 wv = ldg_nc_v4(wr + (size_t)cc * 8);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = __fmaf_rn(lo_bf16(xw[q]), lo_bf16(ww[q]), acc);
      acc = __fmaf_rn(hi_bf16(xw[q]), hi_bf16(ww[q]), acc);
    }
  }
  const float s = warp_fold_sum(acc);
  if (lane == 0) logits[(size_t)t * E + e] = f32_to_bf16(s);
}

// ============================================================== routing
// One warp per token.  Lane j holds logits e = j + 32c.  softmax in fp32 with
// routing_exp and the lane-order sum, gates rounded to bf16, then k rounds of
// a warp-wide max over the key (gate_bits << 16) | (0xFFFF - e), which orders
// by gate descending and expert id ascending.
template <int C>
__global__ void __launch_bounds__(256)
route_topk_kernel(const uint16_t* __restrict__ logits, int T, int E, int k, int norm,
                  int32_t* __restrict__ inds, uint16_t* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const uint16_t* row = logits + (size_t)t * E;
  float v[C];
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    v[c] = bf16_to_f32(row[c * 32 + lane]);
    m = fmaxf(m, v[c]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    v[c] = routing_exp(__fsub_rn(v[c], m));
    s = __fadd_rn(s, v[c]);
  }
  s = warp_fold_sum(s);
  uint32_t key[C];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    uint32_t g = f32_to_bf16(__fdiv_rn(v[c], s));
    key[c] = (g << 16) | (0xFFFFu - static_cast<uint32_t>(c * 32 + lane));
  }
  float ssum = 0.0f;
  uint32_t my_key = 0;  // lane j keeps the j-th selected key
  for (int j = 0; j < k; ++j) {
    uint32_t best = 0;
#pragma unroll
    for (int c = 0; c < C; ++c) best = key[c] > best ? key[c] : best;
    best = __reduce_max_sync(0xffffffffu, best);
    const int e = static_cast<int>(0xFFFFu - (best & 0xFFFFu));
    if ((e & 31) == lane) {
#pragma unroll
      for (int c = 0; c < C; ++c)
        if (c == (e >> 5)) key[c] = 0;
    }
    if (lane == j) my_key = best;
    ssum = __fadd_rn(ssum, bf16_to_f32(static_cast<uint16_t>(best >> 16)));
  }
  if (lane < k) {
    const int e = static_cast<int>(0xFFFFu - (my_key & 0xFFFFu));
    float sc = bf16_to_f32(static_cast<uint16_t>(my_key >> 16));
    if (norm) sc = __fdiv_rn(sc, round_bf16(ssum));
    inds[(size_t)t * k + lane] = e;
    scores[(size_t)t * k + lane] = f32_to_bf16(sc);
  }
}

// ============================================================== dispatch
// Single CTA of 1024 threads.  Shared memory: cnt[E] (pair counts, later the
// scatter cursor) and rank[E] (index of e among the present experts).
constexpr int DSP_THREADS = 1024;

__device__ __forceinline__ int block_excl_scan(int v, int* warp_tot, int* total) {
  // exclusive scan over the block in thread order; returns prefix of v
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int wv = (lane < (blockDim.x >> 5)) ? warp_tot[lane] : 0;
    int wi = wv;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int o = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += o;
    }
    if (lane < (blockDim.x >> 5)) warp_tot[lane] = wi - wv;
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  int r = incl - v + warp_tot[warp];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(DSP_THREADS)
dispatch_kernel(const int32_t* __restrict__ inds, int P, int E, const int32_t* __restrict__ eid2sid,
                int32_t* __restrict__ unique, int32_t* __restrict__ inverse, int32_t* __restrict__ counts,
                int32_t* __restrict__ slot_ids, int32_t* __restrict__ miss_eids,
                int32_t* __restrict__ group_off, int32_t* __restrict__ perm) {
  extern __shared__ int smem_i[];
  int* cnt = smem_i;        // [E]
  int* rank = smem_i + E;   // [E]
  __shared__ int warp_tot[32];
  __shared__ int tot_a, tot_b, tot_c;

  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    int e = inds[p];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();

  // each thread owns a contiguous run of experts [e_lo, e_hi)
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int e_lo = min(E, threadIdx.x * per), e_hi = min(E, e_lo + per);
  int n_present = 0, n_pairs = 0, n_miss = 0;
  for (int e = e_lo; e < e_hi; ++e) {
    if (cnt[e] > 0) {
      ++n_present;
      n_pairs += cnt[e];
      if (eid2sid[e] < 0) ++n_miss;
    }
  }
  int base_u = block_excl_scan(n_present, warp_tot, &tot_a);
  int base_p = block_excl_scan(n_pairs, warp_tot, &tot_b);
  int base_m = block_excl_scan(n_miss, warp_tot, &tot_c);
  for (int e = e_lo; e < e_hi; ++e) {
    int c = cnt[e];
    if (c > 0) {
      int sid = eid2sid[e];
      unique[base_u] = e;
      slot_ids[base_u] = sid;
      group_off[base_u] = base_p;
      if (sid < 0) miss_eids[base_m++] = e;
      rank[e] = base_u++;
      cnt[e] = base_p;  // becomes the scatter cursor
      base_p += c;
    }
  }
  if (threadIdx.x == 0) {
    counts[0] = tot_a;
    counts[1] = tot_c;
    group_off[tot_a] = tot_b;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    int e = inds[p];
    if (e >= 0 && e < E) {
      int pos = atomicAdd(&cnt[e], 1);
      perm[pos] = p;
      inverse[p] = rank[e];
    } else {
      inverse[p] = -1;
    }
  }
}

// ============================================================== fused routing + dispatch
// One launch for softmax / top-k / renormalisation, the expert -> slot lookup
// and the pair permutation.  Phase 1, every CTA: one warp per token, exactly
// the arithmetic of route_topk_kernel; lane j < k also takes the pair's
// position inside its expert's group (an atomicAdd on work[e], the count of
// pairs routed to e so far) and parks it in inverse[p].  Phase 2, the last
// CTA to finish (a ticket in work[E]): a block scan over the per-expert
// counts gives the unique experts in ascending order, their slots, the missed
// ones and the group offsets; every pair then lands at
// perm[group_off[u] + position] and inverse[p] becomes u.  The last CTA
// leaves work[] zero for the next call.
//
// Hand-over: each CTA's pair writes and count atomics precede a GPU-scope
// fence and its ticket atomic; the CTA that draws the last ticket fences again
// and reads the counts, ids and positions through L2 (ld.global.cg), so it
// sees every CTA's writes.
constexpr int RD_WARPS = 32;  // 1024 threads: phase 2 runs on one CTA
constexpr int RD_MAX_E = 1024;

// Optional router trace: the same ids and scores, and the token's raw
// logits, also written to trace memory (typically mapped pinned host memory,
// so they cross PCIe as the kernel produces them; a NULL array is skipped).
struct RouteTrace {
  int32_t* ids;       // [T, k]
  uint16_t* scores;   // [T, k] bf16
  uint16_t* logits;   // [T, E] bf16
};

template <int C>
__global__ void __launch_bounds__(RD_WARPS * 32)
route_dispatch_kernel(const uint16_t* __restrict__ logits, int T, int E, int k, int norm,
                      const int32_t* __restrict__ eid2sid, int32_t* inds, uint16_t* __restrict__ scores,
                      int32_t* __restrict__ unique, int32_t* inverse, int32_t* __restrict__ counts,
                      int32_t* __restrict__ slot_ids, int32_t* __restrict__ miss_eids,
                      int32_t* __restrict__ group_off, int32_t* __restrict__ perm, int32_t* work, RouteTrace tr) {
  __shared__ int s_rank[RD_MAX_E];  // unique index of expert e (phase 2)
  __shared__ int s_base[RD_MAX_E];  // first permutation position of expert e's group
  __shared__ int warp_tot[32];
  __shared__ int tot_a, tot_b, tot_c, s_last;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * RD_WARPS + (threadIdx.x >> 5);
  if (t < T) {
    const uint16_t* row = logits + (size_t)t * E;
    float v[C];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint16_t lb = row[c * 32 + lane];
      if (tr.logits != nullptr) tr.logits[(size_t)t * E + c * 32 + lane] = lb;
      v[c] = bf16_to_f32(lb);
      m = fmaxf(m, v[c]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      v[c] = routing_exp(__fsub_rn(v[c], m));
      s = __fadd_rn(s, v[c]);
    }
    s = warp_fold_sum(s);
    uint32_t key[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      uint32_t g = f32_to_bf16(__fdiv_rn(v[c], s));
      key[c] = (g << 16) | (0xFFFFu - static_cast<uint32_t>(c * 32 + lane));
    }
    float ssum = 0.0f;
    uint32_t my_key = 0;
    for (int j = 0; j < k; ++j) {
      uint32_t best = 0;
#pragma unroll
      for (int c = 0; c < C; ++c) best = key[c] > best ? key[c] : best;
      best = __reduce_max_sync(0xffffffffu, best);
      const int e = static_cast<int>(0xFFFFu - (best & 0xFFFFu));
      if ((e & 31) == lane) {
#pragma unroll
        for (int c = 0; c < C; ++c)
          if (c == (e >> 5)) key[c] = 0;
      }
      if (lane == j) my_key = best;
      ssum = __fadd_rn(ssum, bf16_to_f32(static_cast<uint16_t>(best >> 16)));
    }
    if (lane < k) {
      const int e = static_cast<int>(0xFFFFu - (my_key & 0xFFFFu));
      float sc = bf16_to_f32(static_cast<uint16_t>(my_key >> 16));
      if (norm) sc = __fdiv_rn(sc, round_bf16(ssum));
      const size_t p = (size_t)t * k + lane;
      const uint16_t scb = f32_to_bf16(sc);
      inds[p] = e;
      scores[p] = scb;
      if (tr.ids != nullptr) tr.ids[p] = e;
      if (tr.scores != nullptr) tr.scores[p] = scb;
      inverse[p] = atomicAdd(&work[e], 1);  // position inside the group of e
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&work[E], 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- phase 2, the last CTA: unique / slots / misses / group offsets
  const int P = T * k;
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int e_lo = min(E, (int)threadIdx.x * per), e_hi = min(E, e_lo + per);
  int n_present = 0, n_pairs = 0, n_miss = 0;
  for (int e = e_lo; e < e_hi; ++e) {
    const int c = __ldcg(work + e);
    if (c > 0) {
      ++n_present;
      n_pairs += c;
      if (eid2sid[e] < 0) ++n_miss;
    }
  }
  int base_u = block_excl_scan(n_present, warp_tot, &tot_a);
  int base_p = block_excl_scan(n_pairs, warp_tot, &tot_b);
  int base_m = block_excl_scan(n_miss, warp_tot, &tot_c);
  for (int e = e_lo; e < e_hi; ++e) {
    const int c = __ldcg(work + e);
    if (c > 0) {
      const int sid = eid2sid[e];
      unique[base_u] = e;
      slot_ids[base_u] = sid;
      group_off[base_u] = base_p;
      if (sid < 0) miss_eids[base_m++] = e;
      s_rank[e] = base_u++;
      s_base[e] = base_p;
      base_p += c;
    }
  }
  if (threadIdx.x == 0) {
    counts[0] = tot_a;
    counts[1] = tot_c;
    group_off[tot_a] = tot_b;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = __ldcg(inds + p);
    perm[s_base[e] + __ldcg(inverse + p)] = p;
    inverse[p] = s_rank[e];
  }
  for (int e = threadIdx.x; e <= E; e += blockDim.x) work[e] = 0;  // ready for the next call
}

}  // namespace sg

// ============================================================== C-ABI
extern "C" int sg_router_logits(const uint16_t* x, const uint16_t* w, uint16_t* logits, int T, int H,
                                int E, void* stream) {
  if (T < 0 || E < 1 || H < 256) return SG_ERR_INVALID_ARG;
  if (H % 256 != 0) return SG_ERR_SHAPE;
  if (T == 0) return SG_OK;
  if (!x || !w || !logits) return SG_ERR_INVALID_ARG;
  if (E < sg::RT_WARPS * sg::RT_EXP) {
    const long long warps = (long long)T * E;
    if (warps > (1LL << 30)) return SG_ERR_SHAPE;
    sg::router_logits_small_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(x, w, logits, T, H,
                                                                                                    E);
    SG_LAUNCH_CHECK();
    return SG_OK;
  }
  const size_t smem = (size_t)sg::RT_TOK * H * 2;
  if (smem > 200 * 1024) return SG_ERR_SHAPE;
  static bool attr_done = false;
  if (!attr_done) {
    SG_CUDA_TRY(cudaFuncSetAttribute(sg::router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
    attr_done = true;
  }
  dim3 grid((T + sg::RT_TOK - 1) / sg::RT_TOK, (E + sg::RT_WARPS * sg::RT_EXP - 1) / (sg::RT_WARPS * sg::RT_EXP));
  sg::router_logits_kernel<<<grid, sg::RT_WARPS * 32, smem, (cudaStream_t)stream>>>(x, w, logits, T, H, E);
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_route_topk(const uint16_t* logits, int T, int E, int k, int norm_topk_prob, int32_t* inds,
                             uint16_t* scores, void* stream) {
  if (T < 0) return SG_ERR_INVALID_ARG;
  if (E % 32 != 0 || E < 32 || E > 1024 || k < 1 || k > 32 || k > E) return SG_ERR_SHAPE;
  if (T == 0) return SG_OK;
  if (!logits || !inds || !scores) return SG_ERR_INVALID_ARG;
  const int warps = 8;
  dim3 grid((T + warps - 1) / warps);
  cudaStream_t s = (cudaStream_t)stream;
  const int C = E / 32;
#define SG_ROUTE_CASE(CC) \
  case CC: sg::route_topk_kernel<CC><<<grid, warps * 32, 0, s>>>(logits, T, E, k, norm_topk_prob, inds, scores); break;
  switch (C) {
    SG_ROUTE_CASE(1) SG_ROUTE_CASE(2) SG_ROUTE_CASE(3) SG_ROUTE_CASE(4) SG_ROUTE_CASE(5) SG_ROUTE_CASE(6)
    SG_ROUTE_CASE(7) SG_ROUTE_CASE(8) SG_ROUTE_CASE(9) SG_ROUTE_CASE(10) SG_ROUTE_CASE(11) SG_ROUTE_CASE(12)
    SG_ROUTE_CASE(13) SG_ROUTE_CASE(14) SG_ROUTE_CASE(15) SG_ROUTE_CASE(16) SG_ROUTE_CASE(17)
    SG_ROUTE_CASE(18) SG_ROUTE_CASE(19) SG_ROUTE_CASE(20) SG_ROUTE_CASE(21) SG_ROUTE_CASE(22)
    SG_ROUTE_CASE(23) SG_ROUTE_CASE(24) SG_ROUTE_CASE(25) SG_ROUTE_CASE(26) SG_ROUTE_CASE(27)
    SG_ROUTE_CASE(28) SG_ROUTE_CASE(29) SG_ROUTE_CASE(30) SG_ROUTE_CASE(31) SG_ROUTE_CASE(32)
    default: return SG_ERR_SHAPE;
  }
#undef SG_ROUTE_CASE
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_route_dispatch(const uint16_t* logits, int T, int E, int k, int norm_topk_prob,
                                 const int32_t* eid2sid, int32_t* inds, uint16_t* scores, int32_t* unique,
                                 int32_t* inverse, int32_t* counts, int32_t* slot_ids, int32_t* miss_eids,
                                 int32_t* group_off, int32_t* perm, int max_unique, int32_t* work,
                                 const sg_route_trace* trace, void* stream) {
  if (T < 0) return SG_ERR_INVALID_ARG;
  if (E % 32 != 0 || E < 32 || E > sg::RD_MAX_E || k < 1 || k > 32 || k > E) return SG_ERR_SHAPE;
  if (!eid2sid || !unique || !counts || !slot_ids || !miss_eids || !group_off || !work) return SG_ERR_INVALID_ARG;
  const long long P = (long long)T * k;
  if (P > 0x7FFFFFFFLL) return SG_ERR_SHAPE;
  if (max_unique < (P < E ? (int)P : E) + 1) return SG_ERR_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  if (T == 0) {  // no pairs: an empty dispatch (counts and group_off[0] written)
    SG_CUDA_TRY(cudaMemsetAsync(counts, 0, 2 * sizeof(int32_t), s));
    SG_CUDA_TRY(cudaMemsetAsync(group_off, 0, sizeof(int32_t), s));
    return SG_OK;
  }
  if (!logits || !inds || !scores || !inverse || !perm) return SG_ERR_INVALID_ARG;
  sg::RouteTrace tr{nullptr, nullptr, nullptr};
  if (trace != nullptr) tr = sg::RouteTrace{trace->ids, trace->scores, trace->logits};
  dim3 grid((T + sg::RD_WARPS - 1) / sg::RD_WARPS);
  const int C = E / 32;
#define SG_RD_CASE(CC)                                                                                      \
  case CC:                                                                                                  \
    sg::route_dispatch_kernel<CC><<<grid, sg::RD_WARPS * 32, 0, s>>>(logits, T, E, k, norm_topk_prob,       \
                                                                     eid2sid, inds, scores, unique, inverse, \
                                                                     counts, slot_ids, miss_eids, group_off, \
                                                                     perm, work, tr);                        \
    break;
  switch (C) {
    SG_RD_CASE(1) SG_RD_CASE(2) SG_RD_CASE(3) SG_RD_CASE(4) SG_RD_CASE(5) SG_RD_CASE(6) SG_RD_CASE(7)
    SG_RD_CASE(8) SG_RD_CASE(9) SG_RD_CASE(10) SG_RD_CASE(11) SG_RD_CASE(12) SG_RD_CASE(13) SG_RD_CASE(14)
    SG_RD_CASE(15) SG_RD_CASE(16) SG_RD_CASE(17) SG_RD_CASE(18) SG_RD_CASE(19) SG_RD_CASE(20)
    SG_RD_CASE(21) SG_RD_CASE(22) SG_RD_CASE(23) SG_RD_CASE(24) SG_RD_CASE(25) SG_RD_CASE(26)
    SG_RD_CASE(27) SG_RD_CASE(28) SG_RD_CASE(29) SG_RD_CASE(30) SG_RD_CASE(31) SG_RD_CASE(32)
    default: return SG_ERR_SHAPE;
  }
#undef SG_RD_CASE
  SG_LAUNCH_CHECK();
  return SG_OK;
}

extern "C" int sg_dispatch(const int32_t* inds, int P, int E, const int32_t* eid2sid, int32_t* unique,
                           int32_t* inverse, int32_t* counts, int32_t* slot_ids, int32_t* miss_eids,
                           int32_t* group_off, int32_t* perm, int max_unique, void* stream) {
  if (P < 0 || !eid2sid || !unique || !counts || !slot_ids || !miss_eids || !group_off) return SG_ERR_INVALID_ARG;
  if (P > 0 && (!inds || !inverse || !perm)) return SG_ERR_INVALID_ARG;
  if (E < 1 || E > 8192) return SG_ERR_SHAPE;
  const int need = (P < E ? P : E) + 1;
  if (max_unique < need) return SG_ERR_CAPACITY;
  const size_t smem = (size_t)2 * E * sizeof(int);
  static bool attr_done = false;
  if (!attr_done) {
    SG_CUDA_TRY(cudaFuncSetAttribute(sg::dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
    attr_done = true;
  }
  sg::dispatch_kernel<<<1, sg::DSP_THREADS, smem, (cudaStream_t)stream>>>(inds, P, E, eid2sid, unique, inverse,
                                                                           counts, slot_ids, miss_eids, group_off,
                                                                           perm);
  SG_LAUNCH_CHECK();
  return SG_OK;
}
