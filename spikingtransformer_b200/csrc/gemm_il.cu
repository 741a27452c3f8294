// Fused Linear -> LayerNorm -> LIF, t-coupled rows, T a power of two <= 16.
//
// Same contract as the t-coupled mode of gemm.cu (SSA.py:218-249,
// SpikingMLP.py:31-36, residual adds Encoder.py:19,22 / Decoder.py:18-25),
// organised for epilogue throughput and MMA / epilogue overlap:
//
//  * Tile rows are interleaved token-major: row = tok*T + t.  A permuted 3-D
//    TMA map (dims {K, T, R}, strides {R*K*2, K*2} bytes) writes the 128-row
//    box in that order, so the T timesteps of a token sit in adjacent TMEM
//    lanes of one warp.
//  * Column slices of at most 256 (N = 384 -> 2 x 192, N = 1536 -> 6 x 256,
//    split over a CTA cluster) so two accumulators fit in TMEM: the MMA of
//    tile i+1 runs while the epilogue drains tile i.
//  * Ten warps: warp 0 TMA producer, warp 1 TMEM owner + single-thread
//    tcgen05.mma issuer, warps 2-9 epilogue; each TMEM lane quadrant is read
//    by two epilogue warps, each owning half of the slice's columns.
//  * LayerNorm statistics in one TMEM pass (sums shifted by the first
//    32-column chunk's mean), merged across column halves and cluster CTAs
//    with the parallel-variance formula.
//  * The LIF transposition (lane (tok, t) -> lane (tok, column block)) goes
//    through a warp-private, bank-conflict-free padded shared buffer; the recurrence runs in
//    packed fp32x2 arithmetic (round-to-nearest mul, then add, as the
//    reference) and spikes are written as bf16 bit patterns straight from the
//    threshold compare.
//  * TMEM loads are 32 columns wide and double-buffered.
//  * Compile-time variants: FAST (bf16 spikes and/or residual add only, the
//    residual add specialised) and a general variant for fp32 spikes and the
//    LayerNorm debug output.  The fast variant starts each tile's accumulator
//    with a K = 16 MMA of a ones tile and the bias split into two bf16 terms,
//    folds the LIF input gain into gamma/beta, and runs the LIF branch-free as
//    u = beta (1 - s) u + y + s beta v_reset with s from set.gt.
#include "common.cuh"

namespace spk {
namespace gil {

constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
// the T = 4 epilogue: 16 warps, four groups of one warp per TMEM lane quadrant
// (each accumulator drained by two groups, one per half of the CTA's columns)
constexpr int kEpiWarpsTV = 16;
constexpr int kThreadsTV = 32 * (2 + kEpiWarpsTV);
constexpr int kBK = 64;
constexpr int kAStage = 128 * 128;
constexpr int kMaxSmem = 232448;
// transposition buffer row stride (floats): 16 data + 4 pad, so that both the
// row writes and the transposed reads of a quarter-warp hit 8 distinct bank groups
constexpr int kXS = 20;
// transposed-read epilogue: one staged output box per warp and buffer, [4 t][8 tokens][32 columns] bf16
constexpr int kStgBox = 4 * 8 * 32 * 2;

struct Params {
  int T, tpt;
  int64_t R;
  int K, N, n_cta, cs, num_m_tiles, stages, wbox;
  int res_prefetch;  // the residual rows may be bulk-prefetched (16-byte aligned blocks)
  int nbox;          // T = 4 epilogue: staging boxes per warp
  int epi_warps;     // T = 4 epilogue: 8 or 16 epilogue warps
  int epi;           // epilogue variant (kEpiTranspose, kEpiTV, kEpiTB)
  uint32_t tmem_cols;
  const float *bias, *gamma, *beta_ln;
  float eps;
  const float *lif_beta, *lif_vth, *lif_vr;
  float gain;
  __nv_bfloat16* spk_bf16;
  float* spk_f32;
  __nv_bfloat16* residual;
  float* ln_out;
};

struct Smem {
  uint8_t *a, *w;
  uint8_t *ones, *bsplit;  // fast variant: bias MMA operands (no-swizzle K-major, K = 16)
  float* xs;       // 8 warps x 32 rows x kXS floats (padded rows)
  uint8_t* stg;    // transposed-read epilogue: 8 warps x 2 output boxes (aliases xs)
  uint64_t* rbar;  // transposed-read epilogue: 8 warps x 2 residual-box barriers
  float *bias, *gamma, *beta;
  float2* stat;    // 2 parities x 2 halves x 128 rows (mean, M2)
  float2* xbuf;    // 2 parities x cs x 128 rows (mean, M2)
  float2* mw;      // merge weights: [0] the two column halves, [r] cluster CTA r merged onto 0..r-1
  uint64_t *full, *empty, *acc_full, *acc_empty, *xbar, *drain;
  uint32_t* tmem_base;
  int* abort_flag;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline size_t smem_layout(const Params& p, uint8_t* base, Smem* s) {
  size_t off = 0;
  auto take = [&](size_t bytes, size_t al) {
    off = align_up(off, al);
    size_t o = off;
    off += bytes;
    return o;
  };
  size_t oa = take((size_t)p.stages * kAStage, 1024);
  size_t ow = take((size_t)p.stages * p.n_cta * 128, 1024);
  size_t oon = take(128 * 32, 128), obs = take((size_t)p.n_cta * 32, 128);
  size_t oxs = p.epi == 1   ? take((size_t)p.epi_warps * p.nbox * kStgBox, 1024)
               : p.epi == 0 ? take(kEpiWarps * 32 * kXS * 4, 16)
                            : take((size_t)kEpiWarps * p.T * 2048, 1024);
  size_t ob = take(p.n_cta * 4, 16), og = take(p.n_cta * 4, 16), obe = take(p.n_cta * 4, 16);
  // (mean, M2) of the two column halves: [2 parities][2 halves][128 rows]; the
  // T = 4 epilogue keeps two slots per parity ([2][2 slots][2][128])
  size_t ost = take((size_t)(p.epi == 1 ? 2 : 1) * 2 * 2 * 128 * 8, 16);
  size_t oxb = take((size_t)2 * p.cs * 128 * 8, 16);
  size_t omw = take(16 * 8, 8);
  size_t ofu = take(p.stages * 8, 8), oem = take(p.stages * 8, 8);
  size_t oaf = take(16, 8), oae = take(16, 8), oxbar = take(16, 8), odr = take(8, 8);
  size_t orb = take(kEpiWarpsTV * 2 * 8, 8);
  size_t otm = take(4, 4), oab = take(4, 4);
  if (s) {
    s->a = base + oa;
    s->w = base + ow;
    s->ones = base + oon;
    s->bsplit = base + obs;
    s->xs = reinterpret_cast<float*>(base + oxs);
    s->stg = base + oxs;
    s->rbar = reinterpret_cast<uint64_t*>(base + orb);
    s->bias = reinterpret_cast<float*>(base + ob);
    s->gamma = reinterpret_cast<float*>(base + og);
    s->beta = reinterpret_cast<float*>(base + obe);
    s->stat = reinterpret_cast<float2*>(base + ost);
    s->xbuf = reinterpret_cast<float2*>(base + oxb);
    s->mw = reinterpret_cast<float2*>(base + omw);
    s->full = reinterpret_cast<uint64_t*>(base + ofu);
    s->empty = reinterpret_cast<uint64_t*>(base + oem);
    s->acc_full = reinterpret_cast<uint64_t*>(base + oaf);
    s->acc_empty = reinterpret_cast<uint64_t*>(base + oae);
    s->xbar = reinterpret_cast<uint64_t*>(base + oxbar);
    s->drain = reinterpret_cast<uint64_t*>(base + odr);
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
    s->abort_flag = reinterpret_cast<int*>(base + oab);
  }
  return off;
}

// 1.0f if a > b else 0.0f
__device__ __forceinline__ float set_gt(float a, float b) {
  float r;
  asm("set.gt.f32.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// bf16 pair {hi16(lo), hi16(hi)}: the bf16 patterns of two floats that are 0 or 1
__device__ __forceinline__ uint32_t bf16x2_of_01(float lo, float hi) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(__float_as_uint(lo)), "r"(__float_as_uint(hi)));
  return r;
}

// merge (mean_b, M2_b) over nb samples into (mean, M2) over na samples (parallel-variance
// formula); w = (nb / (na + nb), na * nb / (na + nb)) depends only on the counts, so it is
// computed once per kernel (merge_weights) rather than per row
__device__ __forceinline__ void chan_merge(float& mean, float& m2, float mb, float m2b, float2 w) {
  const float d = mb - mean;
  mean = fmaf(d, w.x, mean);
  m2 = m2 + m2b + d * d * w.y;
}

__device__ __forceinline__ float2 merge_weights(float na, float nb) {
  const float tot = na + nb;
  return make_float2(nb / tot, na * nb / tot);
}

// (mean, M2) of the calling thread's TMEM lane over nch 32-column chunks starting at trow
// (32x32b loads, double-buffered); sums shifted by the row's first value
template <bool DB = true>
__device__ __forceinline__ void lane_row_stats(uint32_t trow, int nch, float inv_cols, float& mean, float& m2) {
  float2 s1a = make_float2(0.0f, 0.0f), s2a = s1a, s1b = s1a, s2b = s1a, nK2 = s1a;
  auto stats_chunk = [&](const uint32_t (&r)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float2 d0 = add2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), nK2);
      const float2 d1 = add2(make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])), nK2);
      s1a = add2(s1a, d0);
      s1b = add2(s1b, d1);
      s2a = fma2(d0, d0, s2a);
      s2b = fma2(d1, d1, s2b);
    }
  };
  float K = 0.0f;
  if constexpr (!DB) {
    // single-buffered (register-lean) form
    for (int c = 0; c < nch; ++c) {
      uint32_t ra[32];
      tmem_ld32_raw(trow + c * 32, ra);
      tmem_wait_ld_fence32(ra);
      if (c == 0) {
        K = __uint_as_float(ra[0]);
        nK2 = make_float2(-K, -K);
      }
      stats_chunk(ra);
    }
  } else {
  uint32_t ra[32], rb[32];
  tmem_ld32_raw(trow, ra);
  for (int c = 0; c < nch; ++c) {
    if ((c & 1) == 0) {
      tmem_wait_ld_fence32(ra);
      if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, rb);
      if (c == 0) {
        K = __uint_as_float(ra[0]);
        nK2 = make_float2(-K, -K);
      }
      stats_chunk(ra);
    } else {
      tmem_wait_ld_fence32(rb);
      if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, ra);
      stats_chunk(rb);
    }
  }
  }
  const float S1 = (s1a.x + s1a.y) + (s1b.x + s1b.y);
  const float S2 = (s2a.x + s2a.y) + (s2b.x + s2b.y);
  mean = K + S1 * inv_cols;
  m2 = fmaxf(S2 - S1 * S1 * inv_cols, 0.0f);
}

// epilogue variants
constexpr int kEpiTranspose = 0;  // rows tok*T + t, lanes transposed through shared memory
constexpr int kEpiTV = 1;         // T = 4, rows t-major within groups of 8 tokens, transposed TMEM reads
constexpr int kEpiTV8 = 3;        // the same with 8 epilogue warps (long K: the tensor cores set the pace)
__host__ __device__ constexpr bool is_tv(int e) { return e == kEpiTV || e == kEpiTV8; }
__host__ __device__ constexpr int tv_warps(int e) { return e == kEpiTV ? kEpiWarpsTV : kEpiWarps; }
constexpr int kEpiTB = 2;         // t-broadcast: rows are tokens, one pre-activation for every step

template <int T, bool FAST, bool RES, int EPI>
__global__ void __launch_bounds__(EPI == kEpiTV ? kThreadsTV : kThreads, 1)
    gemm_il_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmO, const Params p) {
  constexpr int CPL = 16 / T;  // columns per lane after the transposition
  constexpr int TPQ = 32 / T;  // tokens per TMEM lane quadrant
  constexpr int NT = EPI == kEpiTV ? kThreadsTV : kThreads;
  pdl_trigger();
  // dynamic shared memory, 1024-byte aligned (128-byte swizzle atoms); pointers derived from
  // it by plain arithmetic so the compiler keeps them in the shared address space
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  Smem sm;
  smem_layout(p, base, &sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cs = p.cs;
  const uint32_t rank = cs > 1 ? cluster_ctarank() : 0u;
  const int cid = cs > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int ncl = cs > 1 ? (int)cluster_count_x() : (int)gridDim.x;
  const int nk = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], is_tv(EPI) ? tv_warps(EPI) / 2 : EPI == kEpiTB ? kEpiWarps / 2 : kEpiWarps);
      mbar_init(&sm.xbar[i], 1);  // one local arrive (with the expected bytes) per use
    }
    mbar_init(sm.drain, 1);
    if (is_tv(EPI))
      for (int i = 0; i < kEpiWarpsTV * 2; ++i) mbar_init(&sm.rbar[i], 1);
    *sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_base, p.tmem_cols);
    tmem_relinquish();
  }
  if (FAST) {
    // bias as one K = 16 MMA per tile: ones[128 x 16] (columns 0 and 1 = 1) times
    // bsplit[n_cta x 16] (columns 0 and 1 = the bias split into two bf16 terms), both in the
    // no-swizzle K-major layout: 8 x 8 core matrices of 128 bytes, (row, k) at
    // (row / 8) * 256 + (k / 8) * 128 + (row % 8) * 16 + (k % 8) * 2
    const int n0 = (int)rank * p.n_cta;
    for (int i = threadIdx.x; i < 128 * 2; i += NT) {
      const int r = i >> 1, k8 = i & 1;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (k8 == 0) w.x = 0x3F803F80u;  // 1.0, 1.0
      *reinterpret_cast<uint4*>(sm.ones + (r >> 3) * 256 + k8 * 128 + (r & 7) * 16) = w;
    }
    for (int i = threadIdx.x; i < p.n_cta * 2; i += NT) {
      const int r = i >> 1, k8 = i & 1;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (k8 == 0 && p.bias) {
        const float b = p.bias[n0 + r];
        const __nv_bfloat16 hi = __float2bfloat16_rn(b);
        const __nv_bfloat16 lo = __float2bfloat16_rn(b - __bfloat162float(hi));
        w.x = (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
      }
      *reinterpret_cast<uint4*>(sm.bsplit + (r >> 3) * 256 + k8 * 128 + (r & 7) * 16) = w;
    }
    fence_proxy_async_smem();
  }
  {
    // the fast variant folds the LIF input gain into the affine LayerNorm parameters
    const int n0 = (int)rank * p.n_cta;
    const float g = FAST ? p.gain : 1.0f;
    if (threadIdx.x < 16) {
      const int r = threadIdx.x;
      sm.mw[r] = r == 0 ? merge_weights((float)(p.n_cta >> 1), (float)(p.n_cta >> 1))
                        : merge_weights((float)(p.n_cta * r), (float)p.n_cta);
    }
    for (int c = threadIdx.x; c < p.n_cta; c += NT) {
      sm.bias[c] = p.bias ? p.bias[n0 + c] : 0.0f;
      sm.gamma[c] = (p.gamma ? p.gamma[n0 + c] : 1.0f) * g;
      sm.beta[c] = (p.beta_ln ? p.beta_ln[n0 + c] : 0.0f) * g;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (cs > 1) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  // the setup above reads only weights; activations (A, the residual) come after this
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t bytes = (uint32_t)(p.tpt * T * 128) + (uint32_t)p.n_cta * 128;
      const int n0 = (int)rank * p.n_cta;
      bool ok = true;
      uint32_t outstanding = 0, issued_phase = 0;  // bit i: stage i loaded / its phase
      for (int tile = cid; tile < p.num_m_tiles && ok; tile += ncl) {
        if (RES && p.res_prefetch && rank == 0) {
          // the epilogue reads this tile's residual rows about one tile from now: pull them
          // into L2 (one contiguous block of tokens x N per step)
          const int64_t tok0 = (int64_t)tile * p.tpt;
          const int64_t ntok = (p.R - tok0) < p.tpt ? (p.R - tok0) : p.tpt;
          const uint32_t bytes_t = (uint32_t)(ntok * p.N * 2);
          for (int t = 0; t < T; ++t) {
            const __nv_bfloat16* src = p.residual + ((int64_t)t * p.R + tok0) * p.N;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes_t) : "memory");
          }
        }
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1u, 111)) { ok = false; break; }
          outstanding &= ~(1u << stage);
          if (*((volatile int*)sm.abort_flag)) { ok = false; break; }
          mbar_expect_tx(&sm.full[stage], bytes);
          if (is_tv(EPI))  // dims {K, 8 tokens, T, R / 8}: rows g*32 + t*8 + k
            tma_load_4d(sm.a + (size_t)stage * kAStage, &tmA, &sm.full[stage], kc * kBK, 0, 0, tile * 4);
          else if (EPI == kEpiTB)  // dims {K, R}: rows = tokens
            tma_load_2d(sm.a + (size_t)stage * kAStage, &tmA, &sm.full[stage], kc * kBK, tile * 128);
          else
            tma_load_3d(sm.a + (size_t)stage * kAStage, &tmA, &sm.full[stage], kc * kBK, 0, tile * p.tpt);
          uint8_t* w_dst = sm.w + (size_t)stage * p.n_cta * 128;
          for (int r = 0; r < p.n_cta; r += p.wbox)
            tma_load_2d(w_dst + (size_t)r * 128, &tmW, &sm.full[stage], kc * kBK, n0 + r);
          outstanding |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        atomicExch(sm.abort_flag, 1);
        for (int i = 0; i < p.stages; ++i)
          if ((outstanding >> i) & 1u) mbar_wait(&sm.full[i], (issued_phase >> i) & 1u, 112);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int iter = 0;
    for (int tile = cid; tile < p.num_m_tiles && ok; tile += ncl, ++iter) {
      const int buf = iter & 1;
      if (!mbar_wait(&sm.acc_empty[buf], ((uint32_t)(iter >> 1) & 1u) ^ 1u, 121)) { ok = false; break; }
      tc_fence_after();
      const uint32_t dcol = tmem + (uint32_t)(buf * p.n_cta);
      if (FAST && lane == 0)  // accumulator := bias (hi + lo), the K loop accumulates onto it
        umma_bf16(dcol, umma_desc(smem_u32(sm.ones), 128, 256, 0), umma_desc(smem_u32(sm.bsplit), 128, 256, 0),
                  idesc_bf16_f32(128, p.n_cta, 0, 0), 0u);
      for (int kc = 0; kc < nk; ++kc) {
        if (!mbar_wait(&sm.full[stage], phase, 122)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sm.a + (size_t)stage * kAStage);
          const uint32_t w_addr = smem_u32(sm.w + (size_t)stage * p.n_cta * 128);
          const uint32_t idesc = idesc_bf16_f32(128, p.n_cta, 0, 0);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(dcol, umma_desc(a_addr + kk * 32, 16, 1024, 2), umma_desc(w_addr + kk * 32, 16, 1024, 2),
                      idesc, (FAST || (kc | kk)) ? 1u : 0u);
          umma_commit(&sm.empty[stage]);
        }
        __syncwarp();
        if (++stage == p.stages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&sm.acc_full[buf]);
      __syncwarp();
    }
    if (!ok) {
      atomicExch(sm.abort_flag, 1);
      if (lane == 0) umma_commit(sm.drain);
      __syncwarp();
      mbar_wait(sm.drain, 0, 123);
    }
  } else if constexpr (is_tv(EPI)) {
    // ---------------------------------------------------------------- epilogue, transposed TMEM reads
    // Tile rows are ordered q*32 + t*8 + k (k = token within the quadrant's group of 8), so two
    // 16x256b loads at lanes q*32 and q*32 + 16 hand thread i all four steps of token i/4 for the
    // column pairs 8j + 2(i%4): the LIF runs in registers with no transposition.  The spikes of a
    // 32-column chunk are staged with stmatrix as a [t][token][32] box in the 64-byte swizzle and
    // written by one TMA store per warp; with a residual, the box is first loaded by TMA, added to
    // with ldmatrix / stmatrix, and stored back.
    // The epilogue warps form groups of one warp per lane quadrant; group g drains accumulator
    // g % 2 (every other tile of the CTA's sequence).  With 16 warps (short K, where the
    // epilogue sets the pace) group g covers the columns [h n_cta / 2, (h + 1) n_cta / 2), h =
    // g / 2, and a row's statistics are merged over the two halves through shared memory (one
    // named barrier per accumulator) before the cluster merge: four epilogue warps per scheduler
    // hide each other's TMEM, shuffle and arithmetic latencies, and TMEM is read single-buffered.
    // With 8 warps (long K) a group covers all of the CTA's columns and reads TMEM
    // double-buffered.
    static_assert(T == 4 && FAST, "transposed-read epilogue: T = 4, bf16 spikes or residual");
    constexpr int EW = tv_warps(EPI);   // epilogue warps
    constexpr int HALVES = EW / 8;      // groups per accumulator: column halves of the slice
    const int ew = warp - 2;
    const int q = warp & 3;         // TMEM lane quadrant
    const int grp = ew >> 2;        // 0..3
    const int buf = grp & 1;        // accumulator (tile parity) drained by this group
    const int h = grp >> 1;         // column half of the CTA's slice (0 with 8 warps)
    const int tok_l = lane >> 2;    // token within the group of 8
    const int cp = lane & 3;        // column pair within each 8-column group
    const int half = p.n_cta / HALVES;
    const int nch = half / 32;      // this warp's 32-column chunks
    const int c0 = h * half;        // this warp's first column within the CTA's slice
    const int row = q * 32 + lane;  // this lane's tile row in the statistics pass
    const uint32_t lane_lo = (uint32_t)(q * 32) << 16, lane_hi = (uint32_t)(q * 32 + 16) << 16;
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const float2 beta2 = make_float2(beta, beta), nbeta2 = make_float2(-beta, -beta);
    const float bvr = __fmul_rn(beta, vr);
    const float2 bvr2 = make_float2(bvr, bvr);
    const int n0 = (int)rank * p.n_cta + c0;  // this warp's first output column
    const float inv_half = 1.0f / (float)half;
    const float inv_n_all = 1.0f / (float)p.N;
    const float2 w_half = sm.mw[0];
    // this warp's staging boxes (two with a residual: the next chunk's residual box loads while
    // this one is added to; else one); lane i addresses row i%8 of matrix i/8 (8-column group)
    // in the 64-byte swizzle (16-byte unit u of row r at u ^ ((r >> 1) & 3))
    constexpr int NBOX = (EW == 8 || RES) ? 2 : 1;
    constexpr uint32_t kBoxMask = NBOX - 1;
    uint8_t* stg = sm.stg + (size_t)ew * NBOX * kStgBox;
    const int r8 = lane & 7, m8 = lane >> 3;
    const uint32_t mat_off = (uint32_t)(r8 * 64 + ((m8 ^ ((r8 >> 1) & 3)) << 4));
    uint64_t* rbar = sm.rbar + ew * 2;
    uint32_t sc = 0;      // boxes staged so far by this warp (buffer sc & kBoxMask)
    uint32_t rpar = 0;    // bit b: parity of the next residual-box completion on buffer b
    uint32_t rout = 0;    // bit b: a residual box is in flight to buffer b (warp-uniform)
    bool rfail = false;   // a residual box did not land in time: stop waiting for them
    if (lane == 0) tma_prefetch_desc(&tmO);
    int iter = buf;
    for (int tile = cid + buf * ncl; tile < p.num_m_tiles; tile += 2 * ncl, iter += 2) {
      const int y0 = tile * 32 + q * 8;  // first token of this warp's rows
      if (RES && lane == 0) {
        // the tile's first residual box: its latency hides behind the statistics
        const int b = (int)(sc & 1u);
        bulk_wait_read<0>();
        mbar_expect_tx(&rbar[b], (uint32_t)kStgBox);
        tma_load_3d(stg + b * kStgBox, &tmO, &rbar[b], n0, y0, 0);
      }
      if (RES) rout |= 1u << (sc & 1u);
      if (!mbar_wait(&sm.acc_full[buf], (uint32_t)(iter >> 1) & 1u, 131)) { atomicExch(sm.abort_flag, 1); break; }
      tc_fence_after();
      const uint32_t tcol = tmem + (uint32_t)(buf * p.n_cta + c0);
      // ---- statistics: lane l owns tile row q*32 + l (= step l / 8 of token l % 8) over this
      // warp's columns (32x32b loads), sums shifted by the row's first value (the accumulator
      // already holds the bias)
      float mean, m2;
      lane_row_stats<EW == 8>(tcol + lane_lo, nch, inv_half, mean, m2);
      // ---- merge the two column halves (the other group of this accumulator holds the other
      // half); two slots per accumulator, alternating by tile, so a slot is rewritten only after
      // a barrier that every reader of it has passed
      if constexpr (HALVES == 2) {
        float2* st = sm.stat + (size_t)(buf * 2 + ((iter >> 1) & 1)) * 256;
        st[h * 128 + row] = make_float2(mean, m2);
        named_bar_sync(2 + buf, 32 * EW / 2);
        const float2 o = st[(h ^ 1) * 128 + row];
        const float2 a = h == 0 ? make_float2(mean, m2) : o;
        const float2 b = h == 0 ? o : make_float2(mean, m2);
        mean = a.x;
        m2 = a.y;
        chan_merge(mean, m2, b.x, b.y, w_half);
      }
      // ---- merge across the CTAs of the cluster (the row's columns are split over them); the
      // first-half group sends, both groups wait and merge
      if (cs > 1) {
        const int par = buf;
        float2* xb = sm.xbuf + (size_t)par * cs * 128;
        if (h == 0) {
          const uint32_t slot = smem_u32(xb + (size_t)rank * 128 + row);
          const uint32_t bar = smem_u32(&sm.xbar[par]);
          for (int r = 0; r < cs; ++r)
            st_async_f32x2(mapa_shared(slot, (uint32_t)r), mean, m2, mapa_shared(bar, (uint32_t)r));
          if (ew == grp * 4 && lane == 0) mbar_expect_tx(&sm.xbar[par], (uint32_t)(cs * 128 * 8));
        }
        if (!mbar_wait_cluster(&sm.xbar[par], (uint32_t)((iter >> 1) & 1), 132)) {
          atomicExch(sm.abort_flag, 1);
          break;
        }
        float2 a = xb[row];
        mean = a.x;
        m2 = a.y;
        for (int r = 1; r < cs; ++r) {
          const float2 b = xb[(size_t)r * 128 + row];
          chan_merge(mean, m2, b.x, b.y, sm.mw[r]);
        }
      }
      // this lane's row, then the four rows of this thread's token (lanes t*8 + token)
      const float rstd_l = rsqrtf(fmaf(m2, inv_n_all, p.eps));
      const float nmr_l = -mean * rstd_l;
      float2 r2[4], nmr2[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float rstd = __shfl_sync(0xffffffffu, rstd_l, t * 8 + tok_l);
        const float nmr = __shfl_sync(0xffffffffu, nmr_l, t * 8 + tok_l);
        r2[t] = make_float2(rstd, rstd);
        nmr2[t] = make_float2(nmr, nmr);
      }
      // ---- normalise, LIF over t in registers, stage and store one box per 32 columns
      // `next` runs once this chunk's TMEM registers are consumed (before the staging and the
      // store): the single-buffered form issues the next chunk's TMEM loads there
      auto lif_chunk = [&](uint32_t (&lo)[16], uint32_t (&hi)[16], int c, auto&& next) {
        const int b = (int)(sc & kBoxMask);
        uint8_t* box = stg + b * kStgBox;
        const uint32_t box_lane = smem_u32(box) + mat_off;
        uint32_t bits[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = c0 + c * 32 + 8 * j + 2 * cp;
          const float2 g2 = *reinterpret_cast<const float2*>(sm.gamma + col);
          const float2 e2 = *reinterpret_cast<const float2*>(sm.beta + col);
          float2 u = make_float2(0.0f, 0.0f), sp = u;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t* src = (t < 2 ? lo : hi) + 4 * j + 2 * (t & 1);
            float2 y = make_float2(__uint_as_float(src[0]), __uint_as_float(src[1]));
            y = fma2(fma2(y, r2[t], nmr2[t]), g2, e2);
            if (t == 0) {
              u = y;  // membrane starts at 0
            } else {
              y = fma2(sp, bvr2, y);  // exact no-op when v_reset = 0
              u = fma2(fma2(sp, nbeta2, beta2), u, y);
            }
            sp = make_float2(set_gt(u.x, vth), set_gt(u.y, vth));
            bits[t][j] = bf16x2_of_01(sp.x, sp.y);
          }
        }
        next(lo, hi);
        if constexpr (RES) {
          if (!rfail && !mbar_wait(&rbar[b], (rpar >> b) & 1u, 133)) {
            atomicExch(sm.abort_flag, 1);
            rfail = true;
          }
          rpar ^= 1u << b;
          rout &= ~(1u << b);
          if (c + 1 < nch) {
            // the next chunk's residual box into the other buffer, once its last store has read it
            if (lane == 0) {
              bulk_wait_read<0>();
              mbar_expect_tx(&rbar[b ^ 1], (uint32_t)kStgBox);
              tma_load_3d(stg + (b ^ 1) * kStgBox, &tmO, &rbar[b ^ 1], n0 + (c + 1) * 32, y0, 0);
            }
            rout |= 1u << (b ^ 1);
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t rv[4];
            ldmatrix_x4(box_lane + t * 512, rv[0], rv[1], rv[2], rv[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // spikes are exactly 0/1 and the stream holds small integers: the bf16 add is exact
              __nv_bfloat162 x, y;
              *reinterpret_cast<uint32_t*>(&x) = rv[j];
              *reinterpret_cast<uint32_t*>(&y) = bits[t][j];
              const __nv_bfloat162 z = __hadd2(x, y);
              rv[j] = *reinterpret_cast<const uint32_t*>(&z);
            }
            stmatrix_x4(box_lane + t * 512, rv[0], rv[1], rv[2], rv[3]);
          }
        } else {
          if (lane == 0) bulk_wait_read<NBOX - 1>();  // the store that last read this box is done with it
          __syncwarp();
#pragma unroll
          for (int t = 0; t < 4; ++t) stmatrix_x4(box_lane + t * 512, bits[t][0], bits[t][1], bits[t][2], bits[t][3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (y0 < p.R) tma_store_3d(&tmO, box, n0 + c * 32, y0, 0);
          bulk_commit();
        }
        ++sc;
      };
      auto no_next = [](uint32_t (&)[16], uint32_t (&)[16]) {};
      if constexpr (EW == 16) {
        // single-buffered TMEM reads: chunk c + 1 is loaded into the same registers as soon as
        // chunk c's LIF has consumed them, so its latency overlaps chunk c's staging and store
        uint32_t a0[16], a1[16];
        tmem_ld16x256_x4_raw(tcol + lane_lo, a0);
        tmem_ld16x256_x4_raw(tcol + lane_hi, a1);
        for (int c = 0; c < nch; ++c) {
          tmem_wait_ld_fence2(a0, a1);
          if (c + 1 == nch) {
            // last TMEM read of this buffer: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
            lif_chunk(a0, a1, c, no_next);
          } else {
            lif_chunk(a0, a1, c, [&](uint32_t (&lo)[16], uint32_t (&hi)[16]) {
              tmem_ld16x256_x4_raw(tcol + lane_lo + (c + 1) * 32, lo);
              tmem_ld16x256_x4_raw(tcol + lane_hi + (c + 1) * 32, hi);
            });
          }
        }
      } else {
        // double-buffered TMEM reads: chunk c + 1 loads while chunk c is processed
        uint32_t a0[16], a1[16], b0[16], b1[16];
        tmem_ld16x256_x4_raw(tcol + lane_lo, a0);
        tmem_ld16x256_x4_raw(tcol + lane_hi, a1);
        for (int c = 0; c < nch; ++c) {
          if ((c & 1) == 0) {
            tmem_wait_ld_fence2(a0, a1);
            if (c + 1 < nch) {
              tmem_ld16x256_x4_raw(tcol + lane_lo + (c + 1) * 32, b0);
              tmem_ld16x256_x4_raw(tcol + lane_hi + (c + 1) * 32, b1);
            }
          } else {
            tmem_wait_ld_fence2(b0, b1);
            if (c + 1 < nch) {
              tmem_ld16x256_x4_raw(tcol + lane_lo + (c + 1) * 32, a0);
              tmem_ld16x256_x4_raw(tcol + lane_hi + (c + 1) * 32, a1);
            }
          }
          if (c + 1 == nch) {
            // last TMEM read of this buffer: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
          }
          if ((c & 1) == 0)
            lif_chunk(a0, a1, c, no_next);
          else
            lif_chunk(b0, b1, c, no_next);
        }
      }
    }
    // every staged box has been written out (and, with a residual, every load has landed)
    if (lane == 0) bulk_wait<0>();
    if (RES && !rfail) {
      // after an abort a residual box may still be in flight: wait (bounded) for it to land
      for (int b = 0; b < 2; ++b)
        if ((rout >> b) & 1u) mbar_wait(&rbar[b], (rpar >> b) & 1u, 134);
    }
  } else if constexpr (EPI == kEpiTB) {
    // ---------------------------------------------------------------- epilogue, t-broadcast
    // Tile rows are 128 tokens; the same LayerNorm output y drives the LIF at every step
    // (u_t = beta (1 - s) u + y + s beta v_reset), so each lane keeps its token's membrane for a
    // column pair in registers over T.  A 32-column chunk's spikes of all T steps are staged as a
    // warp-private [t][32 tokens][32 columns] box (64-byte swizzle) and written by one TMA store.
    // Two groups of four warps drain alternate tiles (accumulator g), as in the T = 4 epilogue.
    static_assert(FAST && !RES, "t-broadcast epilogue: bf16 spikes only");
    const int ew = warp - 2;
    const int q = warp & 3;
    const int grp = ew >> 2;
    const int nch = p.n_cta / 32;
    const uint32_t lane_lo = (uint32_t)(q * 32) << 16;
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const float2 beta2 = make_float2(beta, beta), nbeta2 = make_float2(-beta, -beta);
    const float bvr = __fmul_rn(beta, vr);
    const float2 bvr2 = make_float2(bvr, bvr);
    const int n0 = (int)rank * p.n_cta;
    const float inv_cta = 1.0f / (float)p.n_cta;
    const float inv_n_all = 1.0f / (float)p.N;
    const int nT = p.T;
    uint8_t* const box = sm.stg + (size_t)ew * nT * 2048;
    if (lane == 0) tma_prefetch_desc(&tmO);
    int iter = grp;
    for (int tile = cid + grp * ncl; tile < p.num_m_tiles; tile += 2 * ncl, iter += 2) {
      const int buf = grp;
      if (!mbar_wait(&sm.acc_full[buf], (uint32_t)(iter >> 1) & 1u, 141)) { atomicExch(sm.abort_flag, 1); break; }
      tc_fence_after();
      const uint32_t trow = tmem + (uint32_t)(buf * p.n_cta) + lane_lo;
      float mean, m2;
      lane_row_stats(trow, nch, inv_cta, mean, m2);
      if (cs > 1) {
        const int par = grp;
        float2* xb = sm.xbuf + (size_t)par * cs * 128;
        const int row = q * 32 + lane;
        const uint32_t slot = smem_u32(xb + (size_t)rank * 128 + row);
        const uint32_t bar = smem_u32(&sm.xbar[par]);
        for (int r = 0; r < cs; ++r)
          st_async_f32x2(mapa_shared(slot, (uint32_t)r), mean, m2, mapa_shared(bar, (uint32_t)r));
        if (ew == grp * 4 && lane == 0) mbar_expect_tx(&sm.xbar[par], (uint32_t)(cs * 128 * 8));
        if (!mbar_wait_cluster(&sm.xbar[par], (uint32_t)((iter >> 1) & 1), 142)) {
          atomicExch(sm.abort_flag, 1);
          break;
        }
        float2 a = xb[row];
        mean = a.x;
        m2 = a.y;
        for (int r = 1; r < cs; ++r) {
          const float2 b = xb[(size_t)r * 128 + row];
          chan_merge(mean, m2, b.x, b.y, sm.mw[r]);
        }
      }
      const float rstd = rsqrtf(fmaf(m2, inv_n_all, p.eps));
      const float2 r2 = make_float2(rstd, rstd);
      const float2 nmr2 = make_float2(-mean * rstd, -mean * rstd);
      const int y0 = tile * 128 + q * 32;  // first token of this warp's rows
      // 8 columns (4 pairs; octet o of the chunk) of this lane's row: normalise, then LIF over
      // every step, each step's 16 bytes into row t*32 + lane of the box
      auto lif_oct = [&](const uint32_t* x, int col, int o) {
        float2 y[4], u[4], sp[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 g2 = *reinterpret_cast<const float2*>(sm.gamma + col + 2 * i);
          const float2 e2 = *reinterpret_cast<const float2*>(sm.beta + col + 2 * i);
          y[i] = fma2(fma2(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), r2, nmr2), g2, e2);
          u[i] = make_float2(0.0f, 0.0f);
          sp[i] = u[i];
        }
#pragma unroll 1
        for (int t = 0; t < nT; ++t) {
          uint32_t bits[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // u = beta (1 - s) u + y + s beta v_reset; at t = 0 u and s are 0, so u = y
            const float2 yy = fma2(sp[i], bvr2, y[i]);
            u[i] = fma2(fma2(sp[i], nbeta2, beta2), u[i], yy);
            sp[i] = make_float2(set_gt(u[i].x, vth), set_gt(u[i].y, vth));
            bits[i] = bf16x2_of_01(sp[i].x, sp[i].y);
          }
          const int row = t * 32 + lane;
          *reinterpret_cast<uint4*>(box + row * 64 + ((o ^ ((row >> 1) & 3)) << 4)) =
              make_uint4(bits[0], bits[1], bits[2], bits[3]);
        }
      };
      uint32_t ra[32], rb[32];
      tmem_ld32_raw(trow, ra);
      for (int c = 0; c < nch; ++c) {
        if ((c & 1) == 0) {
          tmem_wait_ld_fence32(ra);
          if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, rb);
        } else {
          tmem_wait_ld_fence32(rb);
          if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, ra);
        }
        if (c + 1 == nch) {
          // last TMEM read of this buffer: hand it back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
        }
        // the previous chunk's store must have read the box
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if ((c & 1) == 0) {
#pragma unroll
          for (int o = 0; o < 4; ++o) lif_oct(ra + 8 * o, c * 32 + 8 * o, o);
        } else {
#pragma unroll
          for (int o = 0; o < 4; ++o) lif_oct(rb + 8 * o, c * 32 + 8 * o, o);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (y0 < p.R) tma_store_3d(&tmO, box, n0 + c * 32, y0, 0);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp - 2;        // 0..7
    const int q = warp & 3;         // TMEM lane quadrant
    const int h = ew >> 2;          // column half
    const int row = q * 32 + lane;  // tile row = tok * T + t
    const int half = p.n_cta >> 1;
    const float inv_half_o = 1.0f / (float)half;
    const int cb = h * half;        // first column of this warp within the slice
    const int nch = half / 32;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int tok_l = lane / T;     // token within the quadrant
    const int jblk = lane % T;      // timestep (before the transposition) / column block (after)
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const float2 beta2 = make_float2(beta, beta);
    const float2 gain2 = make_float2(p.gain, p.gain);
    const int n0 = (int)rank * p.n_cta;
    const int64_t tstride = p.R * (int64_t)p.N;
    const float inv_n_all = 1.0f / (float)p.N;
    const float2 w_half = sm.mw[0];
    // warp-private transposition buffer: row r (tile row within the quadrant), column c at r*kXS + c
    float* xs = sm.xs + ew * 32 * kXS;
    float* xs_wr = xs + lane * kXS;
    // fast variant: LIF integration as u = beta (1 - s) u + y (+ s beta v_reset), s the previous spike
    const float2 nbeta2 = make_float2(-beta, -beta);
    const float bvr = __fmul_rn(beta, vr);
    const float2 bvr2 = make_float2(bvr, bvr);
    int iter = 0;
    for (int tile = cid; tile < p.num_m_tiles; tile += ncl, ++iter) {
      const int buf = iter & 1;
      if (!mbar_wait(&sm.acc_full[buf], (uint32_t)(iter >> 1) & 1u, 131)) { atomicExch(sm.abort_flag, 1); break; }
      tc_fence_after();
      const uint32_t trow = tmem + lane_off + (uint32_t)(buf * p.n_cta + cb);
      // ---- statistics over this warp's columns
      float mean, m2;
      if constexpr (FAST) {
        // one pass of sums shifted by the row's first value (the bias is already in the accumulator)
        float2 s1a = make_float2(0.0f, 0.0f), s2a = s1a, s1b = s1a, s2b = s1a, nK2 = s1a;
        float K = 0.0f;
        auto stats_chunk = [&](const uint32_t (&r)[32]) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float2 d0 = add2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), nK2);
            const float2 d1 = add2(make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])), nK2);
            s1a = add2(s1a, d0);
            s1b = add2(s1b, d1);
            s2a = fma2(d0, d0, s2a);
            s2b = fma2(d1, d1, s2b);
          }
        };
        uint32_t ra[32], rb[32];
        tmem_ld32_raw(trow, ra);
        for (int c = 0; c < nch; ++c) {
          if ((c & 1) == 0) {
            tmem_wait_ld_fence32(ra);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, rb);
            if (c == 0) {
              K = __uint_as_float(ra[0]);
              nK2 = make_float2(-K, -K);
            }
            stats_chunk(ra);
          } else {
            tmem_wait_ld_fence32(rb);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, ra);
            stats_chunk(rb);
          }
        }
        const float S1 = (s1a.x + s1a.y) + (s1b.x + s1b.y);
        const float S2 = (s2a.x + s2a.y) + (s2b.x + s2b.y);
        const float inv_n = inv_half_o;
        mean = K + S1 * inv_n;
        m2 = fmaxf(S2 - S1 * S1 * inv_n, 0.0f);
      } else {
        float K = 0.0f;
        float2 s1 = make_float2(0.0f, 0.0f), s2 = make_float2(0.0f, 0.0f);
        float2 s1b = s1, s2b = s2;
        auto stats_chunk = [&](const uint32_t (&r)[32], int c) {
          const float* bcol = sm.bias + cb + c * 32;
          if (c == 0) {
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(bcol + i);
              a0 += __uint_as_float(r[i]) + b4.x;
              a1 += __uint_as_float(r[i + 1]) + b4.y;
              a2 += __uint_as_float(r[i + 2]) + b4.z;
              a3 += __uint_as_float(r[i + 3]) + b4.w;
            }
            K = ((a0 + a1) + (a2 + a3)) * (1.0f / 32.0f);
            float q0 = 0.0f, q1 = 0.0f, q2 = 0.0f, q3 = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(bcol + i);
              const float d0 = (__uint_as_float(r[i]) + b4.x) - K, d1 = (__uint_as_float(r[i + 1]) + b4.y) - K;
              const float d2 = (__uint_as_float(r[i + 2]) + b4.z) - K, d3 = (__uint_as_float(r[i + 3]) + b4.w) - K;
              q0 = fmaf(d0, d0, q0);
              q1 = fmaf(d1, d1, q1);
              q2 = fmaf(d2, d2, q2);
              q3 = fmaf(d3, d3, q3);
            }
            s2.x = (q0 + q1) + (q2 + q3);
          } else {
            const float2 nK = make_float2(-K, -K);
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(bcol + i);
              const float2 d0 = add2(add2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])),
                                          make_float2(b4.x, b4.y)), nK);
              const float2 d1 = add2(add2(make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])),
                                          make_float2(b4.z, b4.w)), nK);
              s1 = add2(s1, d0);
              s1b = add2(s1b, d1);
              s2 = fma2(d0, d0, s2);
              s2b = fma2(d1, d1, s2b);
            }
          }
        };
        uint32_t ra[32], rb[32];
        tmem_ld32_raw(trow, ra);
        for (int c = 0; c < nch; ++c) {
          if ((c & 1) == 0) {
            tmem_wait_ld_fence32(ra);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, rb);
            stats_chunk(ra, c);
          } else {
            tmem_wait_ld_fence32(rb);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, ra);
            stats_chunk(rb, c);
          }
        }
        const float S1 = (s1.x + s1.y) + (s1b.x + s1b.y);
        const float S2 = (s2.x + s2.y) + (s2b.x + s2b.y);
        const float inv_n = inv_half_o;
        mean = K + S1 * inv_n;
        m2 = fmaxf(S2 - S1 * S1 * inv_n, 0.0f);
      }
      // ---- merge the two column halves of the slice
      {
        float2* st = sm.stat + (iter & 1) * 256;
        st[h * 128 + row] = make_float2(mean, m2);
        named_bar_sync(1, 32 * kEpiWarps);
        const float2 o = st[(h ^ 1) * 128 + row];
        const float2 a = h == 0 ? make_float2(mean, m2) : o;
        const float2 b = h == 0 ? o : make_float2(mean, m2);
        mean = a.x;
        m2 = a.y;
        chan_merge(mean, m2, b.x, b.y, w_half);
      }
      // ---- merge across the CTAs of the cluster (the row's columns are split over them)
      if (cs > 1) {
        const int par = iter & 1;
        float2* xb = sm.xbuf + (size_t)par * cs * 128;
        if (h == 0) {
          // every row's (mean, M2) into every CTA's slot [rank][row]; the bytes complete the
          // destination's barrier
          const uint32_t slot = smem_u32(xb + (size_t)rank * 128 + row);
          const uint32_t bar = smem_u32(&sm.xbar[par]);
          for (int r = 0; r < cs; ++r)
            st_async_f32x2(mapa_shared(slot, (uint32_t)r), mean, m2, mapa_shared(bar, (uint32_t)r));
        }
        if (threadIdx.x == 64) mbar_expect_tx(&sm.xbar[par], (uint32_t)(cs * 128 * 8));
        if (!mbar_wait_cluster(&sm.xbar[par], (uint32_t)((iter >> 1) & 1), 132)) {
          atomicExch(sm.abort_flag, 1);
          break;
        }
        float2 a = xb[row];
        mean = a.x;
        m2 = a.y;
        for (int r = 1; r < cs; ++r) {
          const float2 b = xb[(size_t)r * 128 + row];
          chan_merge(mean, m2, b.x, b.y, sm.mw[r]);
        }
      }
      const float rstd = rsqrtf(fmaf(m2, inv_n_all, p.eps));
      const float2 rstd2 = make_float2(rstd, rstd);
      const float2 nmean2 = make_float2(-mean, -mean);
      const float nmr = -mean * rstd;
      const float2 nmr2 = make_float2(nmr, nmr);

      // ---- normalise, transpose, LIF, store
      const int64_t gtok = (int64_t)tile * p.tpt + q * TPQ + tok_l;
      const bool tok_ok = gtok < p.R;
      const int64_t lane_out = gtok * p.N + n0 + cb + jblk * CPL;  // element offset at t = 0
      auto norm_sub_fast = [&](const uint32_t* r, int c16) {
        const int col = cb + c16 * 16;  // column within the slice
        const int64_t off0 = lane_out + c16 * 16;
        constexpr int NP = CPL >= 2 ? CPL / 2 : 1;  // bf16 pairs per step
        // residual words of all T steps first: their latency hides behind the arithmetic below
        uint32_t rs[T][NP];
        if (RES && tok_ok) {
#pragma unroll
          for (int t = 0; t < T; ++t) {
            const __nv_bfloat16* src = p.residual + off0 + (int64_t)t * tstride;
            if constexpr (CPL == 16) {
              const uint4 a = *reinterpret_cast<const uint4*>(src), b = *reinterpret_cast<const uint4*>(src + 8);
              rs[t][0] = a.x; rs[t][1] = a.y; rs[t][2] = a.z; rs[t][3] = a.w;
              rs[t][4] = b.x; rs[t][5] = b.y; rs[t][6] = b.z; rs[t][7] = b.w;
            } else if constexpr (CPL == 8) {
              const uint4 a = *reinterpret_cast<const uint4*>(src);
              rs[t][0] = a.x; rs[t][1] = a.y; rs[t][2] = a.z; rs[t][3] = a.w;
            } else if constexpr (CPL == 4) {
              const uint2 a = *reinterpret_cast<const uint2*>(src);
              rs[t][0] = a.x; rs[t][1] = a.y;
            } else if constexpr (CPL == 2) {
              rs[t][0] = *reinterpret_cast<const uint32_t*>(src);
            } else {
              rs[t][0] = *reinterpret_cast<const uint16_t*>(src);
            }
          }
        }
        // (x - mean) rstd before the transposition (per-row statistics; x already holds the
        // bias), gain gamma and gain beta after it (per-column parameters, so each lane loads
        // only its own CPL columns once for all T steps)
        (void)col;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          float2 x0 = make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
          float2 x1 = make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
          x0 = fma2(x0, rstd2, nmr2);
          x1 = fma2(x1, rstd2, nmr2);
          *reinterpret_cast<float4*>(xs_wr + i) = make_float4(x0.x, x0.y, x1.x, x1.y);
        }
        __syncwarp();
        float yt[T][CPL];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int rr = tok_l * T + t;
#pragma unroll
          for (int u = 0; u < CPL; u += (CPL >= 4 ? 4 : CPL)) {
            const float* src = xs + rr * kXS + jblk * CPL + u;
            if constexpr (CPL >= 4) {
              const float4 v4 = *reinterpret_cast<const float4*>(src);
              yt[t][u] = v4.x;
              yt[t][u + 1] = v4.y;
              yt[t][u + 2] = v4.z;
              yt[t][u + 3] = v4.w;
            } else if constexpr (CPL == 2) {
              const float2 v2 = *reinterpret_cast<const float2*>(src);
              yt[t][u] = v2.x;
              yt[t][u + 1] = v2.y;
            } else {
              yt[t][u] = *src;
            }
          }
        }
        __syncwarp();
        if (!tok_ok) return;
        float2 gg[NP], ee[NP];
        {
          const int lc = col + jblk * CPL;  // this lane's first column after the transposition
          float gv[CPL], ev[CPL];
#pragma unroll
          for (int u = 0; u < CPL; u += (CPL >= 4 ? 4 : CPL)) {
            if constexpr (CPL >= 4) {
              const float4 g4 = *reinterpret_cast<const float4*>(sm.gamma + lc + u);
              const float4 e4 = *reinterpret_cast<const float4*>(sm.beta + lc + u);
              gv[u] = g4.x; gv[u + 1] = g4.y; gv[u + 2] = g4.z; gv[u + 3] = g4.w;
              ev[u] = e4.x; ev[u + 1] = e4.y; ev[u + 2] = e4.z; ev[u + 3] = e4.w;
            } else if constexpr (CPL == 2) {
              const float2 g2 = *reinterpret_cast<const float2*>(sm.gamma + lc + u);
              const float2 e2 = *reinterpret_cast<const float2*>(sm.beta + lc + u);
              gv[u] = g2.x; gv[u + 1] = g2.y;
              ev[u] = e2.x; ev[u + 1] = e2.y;
            } else {
              gv[u] = sm.gamma[lc + u];
              ev[u] = sm.beta[lc + u];
            }
          }
#pragma unroll
          for (int u = 0; u < NP; ++u) {
            gg[u] = CPL >= 2 ? make_float2(gv[2 * u], gv[(2 * u + 1) % CPL]) : make_float2(gv[0], 0.0f);
            ee[u] = CPL >= 2 ? make_float2(ev[2 * u], ev[(2 * u + 1) % CPL]) : make_float2(ev[0], 0.0f);
          }
        }
        __nv_bfloat16* sp_ptr = p.spk_bf16 ? p.spk_bf16 + off0 : nullptr;
        float2 u2[NP], s2[NP];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          uint32_t bits[NP];
#pragma unroll
          for (int u = 0; u < NP; ++u) {
            float2 y2 = CPL >= 2 ? make_float2(yt[t][2 * u], yt[t][(2 * u + 1) % CPL]) : make_float2(yt[t][0], 0.0f);
            y2 = fma2(y2, gg[u], ee[u]);
            if (t == 0) {
              u2[u] = y2;  // membrane starts at 0
            } else {
              y2 = fma2(s2[u], bvr2, y2);  // exact no-op when v_reset = 0
              u2[u] = fma2(fma2(s2[u], nbeta2, beta2), u2[u], y2);
            }
            s2[u] = make_float2(set_gt(u2[u].x, vth), set_gt(u2[u].y, vth));
            bits[u] = bf16x2_of_01(s2[u].x, s2[u].y);
          }
          if (sp_ptr) {
            if constexpr (CPL == 16) {
              *reinterpret_cast<uint4*>(sp_ptr) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
              *reinterpret_cast<uint4*>(sp_ptr + 8) = make_uint4(bits[4], bits[5], bits[6], bits[7]);
            } else if constexpr (CPL == 8) {
              *reinterpret_cast<uint4*>(sp_ptr) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
            } else if constexpr (CPL == 4) {
              *reinterpret_cast<uint2*>(sp_ptr) = make_uint2(bits[0], bits[1]);
            } else if constexpr (CPL == 2) {
              *reinterpret_cast<uint32_t*>(sp_ptr) = bits[0];
            } else {
              *reinterpret_cast<uint16_t*>(sp_ptr) = (uint16_t)(bits[0] & 0xFFFFu);
            }
            sp_ptr += tstride;
          }
          if constexpr (RES) {
            // spikes are exactly 0/1 and the stream holds small integers: the bf16 add is exact
            __nv_bfloat16* dst = p.residual + off0 + (int64_t)t * tstride;
            uint32_t o[NP];
#pragma unroll
            for (int u = 0; u < NP; ++u) {
              __nv_bfloat162 a, b;
              *reinterpret_cast<uint32_t*>(&a) = rs[t][u];
              *reinterpret_cast<uint32_t*>(&b) = bits[u];
              const __nv_bfloat162 c = __hadd2(a, b);
              o[u] = *reinterpret_cast<const uint32_t*>(&c);
            }
            if constexpr (CPL == 16) {
              *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
              *reinterpret_cast<uint4*>(dst + 8) = make_uint4(o[4], o[5], o[6], o[7]);
            } else if constexpr (CPL == 8) {
              *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
            } else if constexpr (CPL == 4) {
              *reinterpret_cast<uint2*>(dst) = make_uint2(o[0], o[1]);
            } else if constexpr (CPL == 2) {
              *reinterpret_cast<uint32_t*>(dst) = o[0];
            } else {
              *reinterpret_cast<uint16_t*>(dst) = (uint16_t)(o[0] & 0xFFFFu);
            }
          }
        }
      };
      auto norm_sub = [&](const uint32_t* r, int c16) {
        const int col = cb + c16 * 16;  // column within the slice
        float* ln_dst = nullptr;
        if (!FAST && p.ln_out && tok_ok)
          ln_dst = p.ln_out + (int64_t)(lane % T) * tstride + gtok * p.N + n0 + col;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(sm.bias + col + i);
          const float4 g4 = *reinterpret_cast<const float4*>(sm.gamma + col + i);
          const float4 e4 = *reinterpret_cast<const float4*>(sm.beta + col + i);
          float2 x0 = make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
          float2 x1 = make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
          x0 = add2(add2(x0, make_float2(b4.x, b4.y)), nmean2);
          x1 = add2(add2(x1, make_float2(b4.z, b4.w)), nmean2);
          x0 = fma2(mul2(x0, rstd2), make_float2(g4.x, g4.y), make_float2(e4.x, e4.y));
          x1 = fma2(mul2(x1, rstd2), make_float2(g4.z, g4.w), make_float2(e4.z, e4.w));
          const float4 y4 = make_float4(x0.x, x0.y, x1.x, x1.y);
          *reinterpret_cast<float4*>(xs_wr + i) = y4;
          if (!FAST && ln_dst) *reinterpret_cast<float4*>(ln_dst + i) = y4;
        }
        __syncwarp();
        float yt[T][CPL];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int rr = tok_l * T + t;
#pragma unroll
          for (int u = 0; u < CPL; u += (CPL >= 4 ? 4 : CPL)) {
            const float* src = xs + rr * kXS + jblk * CPL + u;
            if constexpr (CPL >= 4) {
              const float4 v4 = *reinterpret_cast<const float4*>(src);
              yt[t][u] = v4.x;
              yt[t][u + 1] = v4.y;
              yt[t][u + 2] = v4.z;
              yt[t][u + 3] = v4.w;
            } else if constexpr (CPL == 2) {
              const float2 v2 = *reinterpret_cast<const float2*>(src);
              yt[t][u] = v2.x;
              yt[t][u + 1] = v2.y;
            } else {
              yt[t][u] = *src;
            }
          }
        }
        __syncwarp();
        if (!tok_ok) return;
        const int64_t off0 = lane_out + c16 * 16;
        constexpr int NP = CPL >= 2 ? CPL / 2 : 1;  // spike words (bf16 pairs) per step
        float2 mem2[NP];
#pragma unroll
        for (int u = 0; u < NP; ++u) mem2[u] = make_float2(0.0f, 0.0f);
        __nv_bfloat16* sp_ptr = p.spk_bf16 ? p.spk_bf16 + off0 : nullptr;
        // (the general variant is instantiated with RES = true: the pointer is checked at run time)
        __nv_bfloat16* res_ptr = (RES && p.residual) ? p.residual + off0 : nullptr;
#pragma unroll
        for (int t = 0; t < T; ++t) {
          uint32_t bits[NP];
          float sp[CPL];
#pragma unroll
          for (int u = 0; u < NP; ++u) {
            float2 y2 = CPL >= 2 ? make_float2(yt[t][2 * u], yt[t][(2 * u + 1) % CPL]) : make_float2(yt[t][0], 0.0f);
            y2 = mul2(y2, gain2);
            const float2 uu = add2(mul2(mem2[u], beta2), y2);
            const bool f0 = uu.x > vth, f1 = uu.y > vth;
            mem2[u] = make_float2(f0 ? vr : uu.x, f1 ? vr : uu.y);
            bits[u] = (f0 ? 0x3F80u : 0u) | ((CPL >= 2 && f1) ? 0x3F800000u : 0u);
            if (!FAST) {
              sp[(2 * u) % CPL] = f0 ? 1.0f : 0.0f;
              if (CPL >= 2) sp[(2 * u + 1) % CPL] = f1 ? 1.0f : 0.0f;
            }
          }
          if (sp_ptr) {
            if constexpr (CPL == 16) {
              *reinterpret_cast<uint4*>(sp_ptr) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
              *reinterpret_cast<uint4*>(sp_ptr + 8) = make_uint4(bits[4], bits[5], bits[6], bits[7]);
            } else if constexpr (CPL == 8) {
              *reinterpret_cast<uint4*>(sp_ptr) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
            } else if constexpr (CPL == 4) {
              *reinterpret_cast<uint2*>(sp_ptr) = make_uint2(bits[0], bits[1]);
            } else if constexpr (CPL == 2) {
              *reinterpret_cast<uint32_t*>(sp_ptr) = bits[0];
            } else {
              *reinterpret_cast<uint16_t*>(sp_ptr) = (uint16_t)(bits[0] & 0xFFFFu);
            }
            sp_ptr += tstride;
          }
          if (!FAST && p.spk_f32) {
            float* fp = p.spk_f32 + off0 + (int64_t)t * tstride;
#pragma unroll
            for (int u = 0; u < CPL; ++u) fp[u] = sp[u];
          }
          if (RES && res_ptr) {
            // spikes are exactly 0/1 and the stream holds small integers: the bf16 add is exact
#pragma unroll
            for (int u = 0; u < NP; ++u) {
              if (CPL >= 2) {
                __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(res_ptr) + u;
                __nv_bfloat162 sb;
                *reinterpret_cast<uint32_t*>(&sb) = bits[u];
                *r2 = __hadd2(*r2, sb);
              } else {
                __nv_bfloat16 sb;
                *reinterpret_cast<uint16_t*>(&sb) = (uint16_t)(bits[0] & 0xFFFFu);
                *res_ptr = __hadd(*res_ptr, sb);
              }
            }
            res_ptr += tstride;
          }
        }
      };
      if constexpr (FAST) {
        // 16-column TMEM loads, double-buffered
        uint32_t ra[16], rb[16];
        tmem_ld16_raw(trow, ra);
        for (int c = 0; c < 2 * nch; ++c) {
          if ((c & 1) == 0) {
            tmem_wait_ld_fence(ra);
            if (c + 1 < 2 * nch) tmem_ld16_raw(trow + (c + 1) * 16, rb);
          } else {
            tmem_wait_ld_fence(rb);
            if (c + 1 < 2 * nch) tmem_ld16_raw(trow + (c + 1) * 16, ra);
          }
          if (c + 1 == 2 * nch) {
            // last TMEM read of this buffer: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
          }
          if ((c & 1) == 0)
            norm_sub_fast(ra, c);
          else
            norm_sub_fast(rb, c);
        }
      } else {
        uint32_t ra[32], rb[32];
        tmem_ld32_raw(trow, ra);
        for (int c = 0; c < nch; ++c) {
          if ((c & 1) == 0) {
            tmem_wait_ld_fence32(ra);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, rb);
          } else {
            tmem_wait_ld_fence32(rb);
            if (c + 1 < nch) tmem_ld32_raw(trow + (c + 1) * 32, ra);
          }
          if (c + 1 == nch) {
            // last TMEM read of this buffer: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
          }
          if ((c & 1) == 0) {
            norm_sub(ra, 2 * c);
            norm_sub(ra + 16, 2 * c + 1);
          } else {
            norm_sub(rb, 2 * c);
            norm_sub(rb + 16, 2 * c + 1);
          }
        }
      }

    }
  }

  tc_fence_before();
  __syncthreads();
  if (cs > 1) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const Params);

template <int T>
KernelFn pick_kernel(bool fast, bool res, bool tv, bool tv16) {
  if (!fast) return gemm_il_kernel<T, false, true, kEpiTranspose>;
  if constexpr (T == 4) {
    if (tv && tv16) return res ? gemm_il_kernel<4, true, true, kEpiTV> : gemm_il_kernel<4, true, false, kEpiTV>;
    if (tv) return res ? gemm_il_kernel<4, true, true, kEpiTV8> : gemm_il_kernel<4, true, false, kEpiTV8>;
  }
  return res ? gemm_il_kernel<T, true, true, kEpiTranspose> : gemm_il_kernel<T, true, false, kEpiTranspose>;
}

}  // namespace gil

SPK_DEFINE_ERROR_READER(gemm_il_read_device_error)

// Column slice for the interleaved kernel: <= 256 columns (two TMEM
// accumulators), a multiple of 64, at most 8 CTAs per cluster.
bool gemm_il_split(int N, int* cs, int* n_cta) {
  for (int w : {256, 192, 128, 64}) {
    if (N % w == 0 && N / w <= 8) {
      *cs = N / w;
      *n_cta = w;
      return true;
    }
  }
  return false;
}

// Host launcher used by spk_linear_ln_lif_fwd for t-coupled rows with T in
// {1, 2, 4, 8, 16}, and for t-broadcast rows (bf16 spikes, any T); returns
// SPK_ERR_UNSUPPORTED for shapes it does not cover.
int launch_gemm_il(const void* A, const void* W, const float* bias, const float* gamma, const float* beta_ln,
                   float eps, const float* lif_beta, const float* lif_vth, const float* lif_vr, float gain, int T,
                   int64_t R, int K, int N, int t_broadcast, void* spk_bf16, float* spk_f32, void* residual,
                   float* ln_out, cudaStream_t st) {
  using namespace gil;
  if (t_broadcast) {
    if (T > 4 || spk_f32 || ln_out || residual || !spk_bf16 || N % 8 != 0 || !aligned(spk_bf16, 16))
      return SPK_ERR_UNSUPPORTED;
  } else if (!(T == 1 || T == 2 || T == 4 || T == 8 || T == 16)) {
    return SPK_ERR_UNSUPPORTED;
  }
  int cs = 1, n_cta = 0;
  if (!gemm_il_split(N, &cs, &n_cta)) return SPK_ERR_UNSUPPORTED;
  Params p = {};
  p.T = T;
  p.tpt = t_broadcast ? 128 : 128 / T;
  p.R = R;
  p.K = K;
  p.N = N;
  p.n_cta = n_cta;
  p.cs = cs;
  p.num_m_tiles = (int)((R + p.tpt - 1) / p.tpt);
  p.wbox = n_cta;
  p.tmem_cols = 2 * n_cta <= 256 ? 256 : 512;
  p.bias = bias;
  p.gamma = gamma;
  p.beta_ln = beta_ln;
  p.eps = eps;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vr;
  p.gain = gain;
  p.spk_bf16 = reinterpret_cast<__nv_bfloat16*>(spk_bf16);
  p.spk_f32 = spk_f32;
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual);
  p.ln_out = ln_out;
  p.res_prefetch = residual != nullptr && aligned(residual, 16) && N % 8 == 0;
  const bool fast = spk_f32 == nullptr && ln_out == nullptr;
  const bool res = residual != nullptr;
  // the transposed-read epilogue writes one bf16 output (spikes, or the residual stream) by TMA
  void* out = res ? residual : spk_bf16;
  const bool tv = !t_broadcast && T == 4 && fast && R % 8 == 0 && N % 8 == 0 && out != nullptr &&
                  !(res && spk_bf16) && aligned(out, 16);
  p.epi = t_broadcast ? kEpiTB : tv ? kEpiTV : kEpiTranspose;
  // T = 4 epilogue: 16 warps where it sets the pace (K <= 512), else 8 (the deeper operand
  // pipeline that the smaller staging area leaves room for keeps the tensor cores fed)
  const bool tv16 = tv && K <= 512;
  p.epi_warps = tv16 ? kEpiWarpsTV : kEpiWarps;
  p.nbox = tv16 && residual == nullptr ? 1 : 2;

  CUtensorMap tmA, tmW, tmO;
  int rc;
  if (t_broadcast) {
    // dims {K, R}: the box {64, 128} is 128 tokens
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)R};
    uint64_t strides[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {kBK, 128};
    if ((rc = make_tmap_bf16(&tmA, A, 2, dims, strides, box, true)) != SPK_OK) return rc;
    // spikes [T][R][N]: box {32 columns, 32 tokens, T} in the 64-byte swizzle
    uint64_t odims[3] = {(uint64_t)N, (uint64_t)R, (uint64_t)T};
    uint64_t ostrides[2] = {(uint64_t)N * 2, (uint64_t)R * N * 2};
    uint32_t obox[3] = {32, 32, (uint32_t)T};
    if ((rc = make_tmap_bf16_sw(&tmO, spk_bf16, 3, odims, ostrides, obox, 64)) != SPK_OK) return rc;
  } else if (tv) {
    // dims {K, 8, T, R / 8}: the box {64, 8, 4, 4} lands as rows g*32 + t*8 + k, token 8g + k
    uint64_t dims[4] = {(uint64_t)K, 8, (uint64_t)T, (uint64_t)(R / 8)};
    uint64_t strides[3] = {(uint64_t)K * 2, (uint64_t)R * K * 2, (uint64_t)K * 16};
    uint32_t box[4] = {kBK, 8, (uint32_t)T, 4};
    if ((rc = make_tmap_bf16(&tmA, A, 4, dims, strides, box, true)) != SPK_OK) return rc;
    // output [T][R][N]: box {32 columns, 8 tokens, 4 t} in the 64-byte swizzle
    uint64_t odims[3] = {(uint64_t)N, (uint64_t)R, (uint64_t)T};
    uint64_t ostrides[2] = {(uint64_t)N * 2, (uint64_t)R * N * 2};
    uint32_t obox[3] = {32, 8, 4};
    if ((rc = make_tmap_bf16_sw(&tmO, out, 3, odims, ostrides, obox, 64)) != SPK_OK) return rc;
  } else {
    // dims {K, T, R}: the box {64, T, tpt} lands as rows tok*T + t
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)T, (uint64_t)R};
    uint64_t strides[2] = {(uint64_t)R * K * 2, (uint64_t)K * 2};
    uint32_t box[3] = {kBK, (uint32_t)T, (uint32_t)p.tpt};
    if ((rc = make_tmap_bf16(&tmA, A, 3, dims, strides, box, true)) != SPK_OK) return rc;
    tmO = tmA;  // unused
  }
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    uint64_t strides[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {kBK, (uint32_t)p.wbox};
    if ((rc = make_tmap_bf16(&tmW, W, 2, dims, strides, box, true)) != SPK_OK) return rc;
  }
  size_t smem = 0;
  for (p.stages = 4; p.stages >= 2; --p.stages) {
    smem = smem_layout(p, nullptr, nullptr);
    if (smem <= (size_t)kMaxSmem) break;
  }
  if (smem > (size_t)kMaxSmem) return fail(SPK_ERR_SHAPE, "tile of %d columns does not fit in shared memory", n_cta);
  KernelFn kern;
  if (t_broadcast) {
    kern = gemm_il_kernel<1, true, false, kEpiTB>;  // T is read from the parameters
  } else {
    switch (T) {
      case 1: kern = pick_kernel<1>(fast, res, false, false); break;
      case 2: kern = pick_kernel<2>(fast, res, false, false); break;
      case 4: kern = pick_kernel<4>(fast, res, tv, tv16); break;
      case 8: kern = pick_kernel<8>(fast, res, false, false); break;
      default: kern = pick_kernel<16>(fast, res, false, false); break;
    }
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  int clusters = num_sms() / cs;
  if (clusters > p.num_m_tiles) clusters = p.num_m_tiles;
  if (clusters < 1) clusters = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * cs), 1, 1);
  cfg.blockDim = dim3(tv16 ? kThreadsTV : kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cs > 1) {
    // persistent grid: never more clusters than can be co-resident
    int max_clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&max_clusters, (const void*)kern, &cfg) == cudaSuccess && max_clusters > 0 &&
        max_clusters < clusters) {
      clusters = max_clusters;
      cfg.gridDim = dim3((unsigned)(clusters * cs), 1, 1);
    }
  }
  add_pdl_attr(cfg, attr);  // after the occupancy query, which describes the cluster shape alone
  e = cudaLaunchKernelEx(&cfg, kern, tmA, tmW, tmO, p);
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "gemm_il_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

}  // namespace spk
