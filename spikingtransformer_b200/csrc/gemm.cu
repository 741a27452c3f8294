// Fused Linear -> LayerNorm -> LIF on the 5th-generation tensor cores.
//
// Reference composition (flofiz/SpikingTransformer):
//   SSA.py:218-228, :247-249   q/k/v/out_proj -> LayerNorm -> LIF
//   SpikingMLP.py:26-37        expand -> LN -> LIF, compress -> LN -> LIF
//   Encoder.py:19,22 / Decoder.py:18-25   residual add of the spike output
//   Seq2Seq.py:117             output_layer (plain Linear)
//
// One persistent kernel, three epilogues:
//   MODE_TCOUPLED  A is [T][R][K] (t-major fold).  A 128-row tile holds
//                  tpt = floor(128/T) tokens at all T timesteps (rows
//                  t*tpt + tok), loaded by one 3-D TMA box, so the LIF
//                  recurrence over t stays inside the CTA.
//   MODE_TBCAST    A is [R][K]; the same pre-activation is fed to the LIF at
//                  every step (the T-fold of an input repeated over t,
//                  Seq2Seq.py:101 + the patch embedding).
//   MODE_PLAIN     y = A W^T + b in fp32 (output layer).
//
// Warp roles (192 threads): warp 0 issues TMA loads into a ring of shared
// memory stages; warp 1 owns the TMEM allocation and one elected thread
// issues tcgen05.mma (bf16 x bf16 -> fp32 in TMEM, 128 x n_cta per tile);
// warps 2-5 are the epilogue, one TMEM lane (= tile row) per thread.
//
// LayerNorm: each CTA holds its n_cta columns of the 128 rows in TMEM.  Rows
// wider than one CTA (N > 512, e.g. the 1536-wide MLP expansion) are split
// over a cluster of cs CTAs; each computes per-row (sum, centred sum of
// squares) over its slice, pushes them into every peer's shared memory
// (st.shared::cluster + remote mbarrier arrive) and combines them with the
// parallel-variance formula.  Pre-activations never leave the SM.
//
// LIF (MODE_TCOUPLED): the normalised 32-column chunk of all 128 rows is
// staged in shared memory, then each thread runs the recurrence over t for
// two columns of one token and writes bf16 (or fp32) spikes, optionally
// adding them into the residual stream in place.
#include <cstdlib>

#include "common.cuh"

namespace spk {
namespace gemmk {

enum { MODE_TCOUPLED = 0, MODE_TBCAST = 1, MODE_PLAIN = 2 };

constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kBK = 64;                 // K elements per stage (128 bytes of bf16)
constexpr int kAStageBytes = 128 * 128; // 128 rows x 128 B
constexpr int kYsStride = 36;           // floats per staged row (32 + pad)
constexpr int kMaxSmem = 232448;        // sm_100 opt-in limit per block

struct Params {
  int T, tpt;
  int64_t R;        // rows per timestep (TCOUPLED) / rows (others)
  int K, N;
  int n_cta;        // columns per CTA tile
  int cs;           // cluster size (LN split), 1 if none
  int num_m_tiles, num_n_tiles;
  int stages;
  int wbox;         // rows per W TMA box
  uint32_t tmem_cols;
  const float* bias;
  const float* gamma;
  const float* beta_ln;
  float eps;
  const float* lif_beta;
  const float* lif_vth;
  const float* lif_vr;
  float gain;
  __nv_bfloat16* spk_bf16;  // [T][R][N]
  float* spk_f32;           // [T][R][N]
  __nv_bfloat16* residual;  // [T][R][N] (+= spikes)
  float* ln_out;            // TCOUPLED: [T][R][N]; TBCAST: [R][N]
  float* out_f32;           // PLAIN: [R][N]
  int vec_out;              // PLAIN: N % 4 == 0 and out, bias 16-byte aligned
  int norm;                 // TCOUPLED / TBCAST: 1 LayerNorm over the N features, 0 per-feature affine only
  // PLAIN only: operand layouts and split K
  int a_mn;                 // A stored [K][M] (contiguous along M) instead of [M][K]
  int b_mn;                 // W stored [K][N] (contiguous along N) instead of [N][K]
  int k_splits;             // the K blocks are split over this many tiles, each writing partial sums
  int kb_per_split;         // K blocks (of kBK) per split
  int64_t split_stride;     // elements between the outputs of consecutive splits
  int nacc;                 // TMEM accumulators (2: the MMA of tile i+1 runs while the epilogue drains tile i)
};

struct Smem {
  uint8_t* a;      // stages x 16 KB
  uint8_t* w;      // stages x n_cta*128 B
  float* ys;       // 128 x kYsStride
  float* bias;     // n_cta
  float* gamma;    // n_cta
  float* beta;     // n_cta
  float* xbuf;     // 2 x cs x 128 x 2
  uint64_t* full;  // stages
  uint64_t* empty; // stages
  uint64_t* acc_full;
  uint64_t* acc_empty;
  uint64_t* xbar;  // 2
  uint64_t* drain;
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
  size_t oa = take((size_t)p.stages * kAStageBytes, 1024);
  size_t ow = take((size_t)p.stages * p.n_cta * 128, 1024);
  size_t oys = take(128 * kYsStride * 4, 16);
  size_t ob = take(p.n_cta * 4, 16);
  size_t og = take(p.n_cta * 4, 16);
  size_t obe = take(p.n_cta * 4, 16);
  size_t ox = take((size_t)2 * p.cs * 128 * 2 * 4, 16);
  size_t ofull = take(p.stages * 8, 8);
  size_t oempty = take(p.stages * 8, 8);
  size_t oaf = take(16, 8), oae = take(16, 8), oxb = take(16, 8), odr = take(8, 8);
  size_t otm = take(4, 4), oab = take(4, 4);
  if (s) {
    s->a = base + oa;
    s->w = base + ow;
    s->ys = reinterpret_cast<float*>(base + oys);
    s->bias = reinterpret_cast<float*>(base + ob);
    s->gamma = reinterpret_cast<float*>(base + og);
    s->beta = reinterpret_cast<float*>(base + obe);
    s->xbuf = reinterpret_cast<float*>(base + ox);
    s->full = reinterpret_cast<uint64_t*>(base + ofull);
    s->empty = reinterpret_cast<uint64_t*>(base + oempty);
    s->acc_full = reinterpret_cast<uint64_t*>(base + oaf);
    s->acc_empty = reinterpret_cast<uint64_t*>(base + oae);
    s->xbar = reinterpret_cast<uint64_t*>(base + oxb);
    s->drain = reinterpret_cast<uint64_t*>(base + odr);
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
    s->abort_flag = reinterpret_cast<int*>(base + oab);
  }
  return off + 1024;  // slack for aligning the dynamic base
}

__device__ __forceinline__ void lif_step(float y, float gain, float beta, float vth, float vr, float& v, float& s) {
  const float cur = gain != 1.0f ? __fmul_rn(y, gain) : y;
  const float u = __fadd_rn(__fmul_rn(v, beta), cur);
  const bool fire = u > vth;
  s = fire ? 1.0f : 0.0f;
  v = fire ? vr : u;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_ln_lif_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const Params p) {
  // dynamic shared memory, 1024-byte aligned (128-byte swizzle atoms); pointers derived from
  // it by plain arithmetic so the compiler keeps them in the shared address space
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  Smem sm;
  smem_layout(p, base, &sm);
  pdl_trigger();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cs = p.cs;
  const uint32_t rank = cs > 1 ? cluster_ctarank() : 0u;
  const int cid = cs > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int ncl = cs > 1 ? (int)cluster_count_x() : (int)gridDim.x;
  const int mn_tiles = p.num_m_tiles * p.num_n_tiles;
  const int ksplits = (MODE == MODE_PLAIN && p.k_splits > 1) ? p.k_splits : 1;
  const int total_tiles = mn_tiles * ksplits;
  const int nk = (p.K + kBK - 1) / kBK;
  // K blocks [kc_lo, kc_hi) of a tile (split K: tile / mn_tiles is the split)
  auto k_range = [&](int tile, int& kc_lo, int& kc_hi) {
    if (ksplits > 1) {
      kc_lo = (tile / mn_tiles) * p.kb_per_split;
      kc_hi = min(nk, kc_lo + p.kb_per_split);
    } else {
      kc_lo = 0;
      kc_hi = nk;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiThreads);
    }
    mbar_init(&sm.xbar[0], 4 * cs);
    mbar_init(&sm.xbar[1], 4 * cs);
    mbar_init(sm.drain, 1);
    *sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_base, p.tmem_cols);
    tmem_relinquish();
  }
  // per-CTA column parameters (LN modes: the slice is fixed for the CTA)
  if (MODE != MODE_PLAIN) {
    const int n0 = (int)rank * p.n_cta;
    for (int c = threadIdx.x; c < p.n_cta; c += kThreads) {
      sm.bias[c] = p.bias ? p.bias[n0 + c] : 0.0f;
      sm.gamma[c] = p.gamma ? p.gamma[n0 + c] : 1.0f;
      sm.beta[c] = p.beta_ln ? p.beta_ln[n0 + c] : 0.0f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (cs > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  // the setup above reads only weights and constants; activations come after this
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t a_bytes = (MODE == MODE_TCOUPLED) ? (uint32_t)(p.tpt * p.T * 128) : (uint32_t)kAStageBytes;
      const uint32_t w_bytes = (uint32_t)p.n_cta * 128;
      bool ok = true;
      int outstanding[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint32_t issued_phase[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int tile = cid; tile < total_tiles && ok; tile += ncl) {
        const int tmn = tile % mn_tiles;
        const int mt = tmn / p.num_n_tiles;
        const int n0 = (MODE == MODE_PLAIN) ? (tmn % p.num_n_tiles) * p.n_cta : (int)rank * p.n_cta;
        int kc_lo, kc_hi;
        k_range(tile, kc_lo, kc_hi);
        for (int kc = kc_lo; kc < kc_hi; ++kc) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1u, 11)) { ok = false; break; }
          outstanding[stage] = 0;
          if (*((volatile int*)sm.abort_flag)) { ok = false; break; }
          mbar_expect_tx(&sm.full[stage], a_bytes + w_bytes);
          uint8_t* a_dst = sm.a + (size_t)stage * kAStageBytes;
          if (MODE == MODE_TCOUPLED) {
            tma_load_3d(a_dst, &tmA, &sm.full[stage], kc * kBK, mt * p.tpt, 0);
          } else if (MODE == MODE_PLAIN && p.a_mn) {
            // A [K][M]: two 64 (m) x 64 (k) atoms, 128-byte rows along m
            tma_load_2d(a_dst, &tmA, &sm.full[stage], mt * 128, kc * kBK);
            tma_load_2d(a_dst + 8192, &tmA, &sm.full[stage], mt * 128 + 64, kc * kBK);
          } else {
            tma_load_2d(a_dst, &tmA, &sm.full[stage], kc * kBK, mt * 128);
          }
          uint8_t* w_dst = sm.w + (size_t)stage * p.n_cta * 128;
          if (MODE == MODE_PLAIN && p.b_mn) {
            // W [K][N]: n_cta / 64 atoms of 64 (n) x 64 (k)
            for (int j = 0; j < p.n_cta; j += 64)
              tma_load_2d(w_dst + (size_t)j * 128, &tmW, &sm.full[stage], n0 + j, kc * kBK);
          } else {
            for (int r = 0; r < p.n_cta; r += p.wbox)
              tma_load_2d(w_dst + (size_t)r * 128, &tmW, &sm.full[stage], kc * kBK, n0 + r);
          }
          outstanding[stage] = 1;
          issued_phase[stage] = phase;
          if (++stage == p.stages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        atomicExch(sm.abort_flag, 1);
        // drain loads still in flight before the CTA may exit
        for (int i = 0; i < p.stages; ++i)
          if (outstanding[i]) mbar_wait(&sm.full[i], issued_phase[i], 12);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    const int nsub_max = 256;
    const int amn = (MODE == MODE_PLAIN) ? p.a_mn : 0, bmn = (MODE == MODE_PLAIN) ? p.b_mn : 0;
    for (int tile = cid; tile < total_tiles && ok; tile += ncl, ++it) {
      const int abuf = p.nacc == 2 ? (it & 1) : 0;
      const uint32_t aph = (uint32_t)(p.nacc == 2 ? (it >> 1) : it) & 1u;
      if (!mbar_wait(&sm.acc_empty[abuf], aph ^ 1u, 21)) { ok = false; break; }
      tc_fence_after();
      const uint32_t dacc = tmem + (uint32_t)(abuf * p.n_cta);
      int kc_lo, kc_hi;
      k_range(tile, kc_lo, kc_hi);
      for (int kc = kc_lo; kc < kc_hi; ++kc) {
        if (!mbar_wait(&sm.full[stage], phase, 22)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sm.a + (size_t)stage * kAStageBytes);
          const uint32_t w_addr = smem_u32(sm.w + (size_t)stage * p.n_cta * 128);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major operands advance 16 elements (32 bytes) along the 128-byte row per
            // K step; MN-major ones advance 16 rows (2048 bytes), their 64-wide MN atoms
            // 8192 bytes apart
            const uint64_t adesc = amn ? umma_desc(a_addr + kk * 2048, 8192, 1024, 2)
                                       : umma_desc(a_addr + kk * 32, 16, 1024, 2);
            for (int nb = 0; nb < p.n_cta; nb += nsub_max) {
              const int nsz = min(nsub_max, p.n_cta - nb);
              const uint64_t bdesc = bmn ? umma_desc(w_addr + (nb / 64) * 8192 + kk * 2048, 8192, 1024, 2)
                                         : umma_desc(w_addr + nb * 128 + kk * 32, 16, 1024, 2);
              umma_bf16(dacc + nb, adesc, bdesc, idesc_bf16_f32(128, nsz, amn, bmn),
                        (kc != kc_lo || kk) ? 1u : 0u);
            }
          }
          umma_commit(&sm.empty[stage]);
        }
        __syncwarp();
        if (++stage == p.stages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&sm.acc_full[abuf]);
      __syncwarp();
    }
    if (!ok) {
      atomicExch(sm.abort_flag, 1);
      // all MMAs issued so far complete before TMEM is released
      if (lane == 0) umma_commit(sm.drain);
      __syncwarp();
      mbar_wait(sm.drain, 0, 23);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    const int etid = threadIdx.x - 64;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const float beta = p.lif_beta ? __ldg(p.lif_beta) : 0.0f;
    const float vth = p.lif_vth ? __ldg(p.lif_vth) : 0.0f;
    const float vr = p.lif_vr ? __ldg(p.lif_vr) : 0.0f;
    float bsum = 0.0f;
    if (MODE != MODE_PLAIN)
      for (int c = 0; c < p.n_cta; ++c) bsum += sm.bias[c];
    int iter = 0;
    for (int tile = cid; tile < total_tiles; tile += ncl, ++iter) {
      const int abuf = p.nacc == 2 ? (iter & 1) : 0;
      const uint32_t aph = (uint32_t)(p.nacc == 2 ? (iter >> 1) : iter) & 1u;
      if (!mbar_wait(&sm.acc_full[abuf], aph, 31)) { atomicExch(sm.abort_flag, 1); break; }
      tc_fence_after();
      const uint32_t tacc = trow + (uint32_t)(abuf * p.n_cta);  // this thread's lane of the tile's accumulator
      const int mt = (tile % mn_tiles) / p.num_n_tiles;

      if (MODE == MODE_PLAIN) {
        const int n0 = ((tile % mn_tiles) % p.num_n_tiles) * p.n_cta;
        const int64_t grow = (int64_t)mt * 128 + row;
        // split K: split s writes its partial sums s * split_stride further on; the
        // bias goes into split 0 only
        const int split = tile / mn_tiles;
        float* outp = p.out_f32 + (int64_t)split * p.split_stride;
        const float* biasp = split == 0 ? p.bias : nullptr;
        for (int c0 = 0; c0 < p.n_cta; c0 += 32) {
          float v[32];
          tmem_ld32(tacc + c0, v);
          tmem_wait_ld();
          if (p.vec_out) {
            // transpose through the warp's 32 staged rows so that every store
            // instruction writes four 128-byte row segments
            float* ys = sm.ys + row * kYsStride;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(ys + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            __syncwarp();
            const int cb = n0 + c0 + 4 * (lane & 7);
            float4 b4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (biasp && cb < p.N) b4 = __ldg(reinterpret_cast<const float4*>(biasp + cb));
            const float* ysw = sm.ys + q * 32 * kYsStride + 4 * (lane & 7);
            const int64_t rbase = (int64_t)mt * 128 + q * 32;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int r = 4 * k + (lane >> 3);
              const float4 y = *reinterpret_cast<const float4*>(ysw + r * kYsStride);
              if (rbase + r < p.R && cb < p.N)
                *reinterpret_cast<float4*>(outp + (rbase + r) * p.N + cb) =
                    make_float4(y.x + b4.x, y.y + b4.y, y.z + b4.z, y.w + b4.w);
            }
            __syncwarp();
          } else if (grow < p.R) {
            float* dst = outp + grow * p.N + n0 + c0;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = n0 + c0 + i;
              if (col < p.N) dst[i] = v[i] + (biasp ? __ldg(biasp + col) : 0.0f);
            }
          }
        }
      } else {
        // ---- LayerNorm statistics (none for the affine-only epilogue: mean 0, rstd 1)
        float mean = 0.0f, rstd = 1.0f;
        if (p.norm) {
          float s = 0.0f;
          for (int c0 = 0; c0 < p.n_cta; c0 += 32) {
            float v[32];
            tmem_ld32(tacc + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) s += v[i];
          }
          const float xsum = s + bsum;
          const float m_loc = xsum / (float)p.n_cta;
          float m2 = 0.0f;
          for (int c0 = 0; c0 < p.n_cta; c0 += 32) {
            float v[32];
            tmem_ld32(tacc + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = (v[i] + sm.bias[c0 + i]) - m_loc;
              m2 = fmaf(d, d, m2);
            }
          }
          mean = m_loc;
          float var = m2 / (float)p.n_cta;
          if (cs > 1) {
            const int par = iter & 1;
            float* xb = sm.xbuf + (size_t)par * cs * 128 * 2;
            const uint32_t my_slot = smem_u32(xb + ((size_t)rank * 128 + row) * 2);
            for (int r = 0; r < cs; ++r) st_cluster_f32x2(mapa_shared(my_slot, (uint32_t)r), xsum, m2);
            fence_acq_rel_cluster();
            __syncwarp();
            if (lane == 0)
              for (int r = 0; r < cs; ++r) mbar_arrive_remote(mapa_shared(smem_u32(&sm.xbar[par]), (uint32_t)r));
            if (!mbar_wait_cluster(&sm.xbar[par], (uint32_t)((iter >> 1) & 1), 32)) {
              atomicExch(sm.abort_flag, 1);
              break;
            }
            float tot = 0.0f;
            for (int r = 0; r < cs; ++r) tot += xb[((size_t)r * 128 + row) * 2];
            mean = tot / (float)p.N;
            float M2 = 0.0f;
            for (int r = 0; r < cs; ++r) {
              const float sr = xb[((size_t)r * 128 + row) * 2];
              const float m2r = xb[((size_t)r * 128 + row) * 2 + 1];
              const float dm = sr / (float)p.n_cta - mean;
              M2 += m2r + (float)p.n_cta * dm * dm;
            }
            var = M2 / (float)p.N;
          }
          rstd = 1.0f / sqrtf(var + p.eps);
        }
        const int n0 = (int)rank * p.n_cta;

        if (MODE == MODE_TCOUPLED) {
          const int t_row = row / p.tpt, tok_row = row - t_row * p.tpt;
          const int64_t tok_base = (int64_t)mt * p.tpt;
          const bool row_valid = t_row < p.T && tok_base + tok_row < p.R;
          const int pairs = p.tpt * 16;
          for (int c0 = 0; c0 < p.n_cta; c0 += 32) {
            float v[32];
            tmem_ld32(tacc + c0, v);
            tmem_wait_ld();
            float* ys = sm.ys + row * kYsStride;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = (v[i] + sm.bias[c0 + i]) - mean;
              v[i] = fmaf(d * rstd, sm.gamma[c0 + i], sm.beta[c0 + i]);
            }
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(ys + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (p.ln_out && row_valid) {
              float* dst = p.ln_out + ((int64_t)t_row * p.R + tok_base + tok_row) * p.N + n0 + c0;
#pragma unroll
              for (int i = 0; i < 32; ++i) dst[i] = v[i];
            }
            named_bar_sync(1, kEpiThreads);
            for (int pi = etid; pi < pairs; pi += kEpiThreads) {
              const int tok = pi >> 4;
              const int col = (pi & 15) * 2;
              const int64_t gtok = tok_base + tok;
              if (gtok >= p.R) continue;
              float v0 = 0.0f, v1 = 0.0f;
              for (int t = 0; t < p.T; ++t) {
                const float2 y = *reinterpret_cast<const float2*>(sm.ys + (t * p.tpt + tok) * kYsStride + col);
                float s0, s1;
                lif_step(y.x, p.gain, beta, vth, vr, v0, s0);
                lif_step(y.y, p.gain, beta, vth, vr, v1, s1);
                const int64_t o = ((int64_t)t * p.R + gtok) * p.N + n0 + c0 + col;
                if (p.spk_bf16) *reinterpret_cast<__nv_bfloat162*>(p.spk_bf16 + o) = __floats2bfloat162_rn(s0, s1);
                if (p.spk_f32) *reinterpret_cast<float2*>(p.spk_f32 + o) = make_float2(s0, s1);
                if (p.residual) {
                  __nv_bfloat162* rp = reinterpret_cast<__nv_bfloat162*>(p.residual + o);
                  const float2 r = __bfloat1622float2(*rp);
                  *rp = __floats2bfloat162_rn(r.x + s0, r.y + s1);
                }
              }
            }
            named_bar_sync(1, kEpiThreads);
          }
        } else {  // MODE_TBCAST
          const int64_t gtok = (int64_t)mt * 128 + row;
          for (int c0 = 0; c0 < p.n_cta; c0 += 32) {
            float v[32];
            tmem_ld32(tacc + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = (v[i] + sm.bias[c0 + i]) - mean;
              v[i] = fmaf(d * rstd, sm.gamma[c0 + i], sm.beta[c0 + i]);
            }
            if (gtok < p.R) {
              if (p.ln_out) {
                float* dst = p.ln_out + gtok * p.N + n0 + c0;
#pragma unroll
                for (int i = 0; i < 32; ++i) dst[i] = v[i];
              }
              float mem[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) mem[i] = 0.0f;
              for (int t = 0; t < p.T; ++t) {
                const int64_t o = ((int64_t)t * p.R + gtok) * p.N + n0 + c0;
                float sp[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) lif_step(v[i], p.gain, beta, vth, vr, mem[i], sp[i]);
                if (p.spk_bf16) {
#pragma unroll
                  for (int i = 0; i < 32; i += 2)
                    *reinterpret_cast<__nv_bfloat162*>(p.spk_bf16 + o + i) = __floats2bfloat162_rn(sp[i], sp[i + 1]);
                }
                if (p.spk_f32) {
#pragma unroll
                  for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4*>(p.spk_f32 + o + i) = make_float4(sp[i], sp[i + 1], sp[i + 2], sp[i + 3]);
                }
                if (p.residual) {
#pragma unroll
                  for (int i = 0; i < 32; i += 2) {
                    __nv_bfloat162* rp = reinterpret_cast<__nv_bfloat162*>(p.residual + o + i);
                    const float2 r = __bfloat1622float2(*rp);
                    *rp = __floats2bfloat162_rn(r.x + sp[i], r.y + sp[i + 1]);
                  }
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[abuf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (cs > 1) cluster_sync_all();  // no peer may still write into this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

}  // namespace gemmk

SPK_DEFINE_ERROR_READER(gemm_read_device_error)

using namespace gemmk;

static int launch_gemm_maps(int mode, const CUtensorMap& tmA, const CUtensorMap& tmW, Params& p, cudaStream_t st);
static uint32_t tmem_cols_for(int n);

static int launch_gemm(int mode, const void* A, const void* W, Params& p, int64_t T_rows, cudaStream_t st) {
  // ---- tensor maps
  CUtensorMap tmA, tmW;
  int rc;
  if (mode == MODE_TCOUPLED) {
    uint64_t dims[3] = {(uint64_t)p.K, (uint64_t)p.R, (uint64_t)p.T};
    uint64_t strides[2] = {(uint64_t)p.K * 2, (uint64_t)p.R * p.K * 2};
    uint32_t box[3] = {kBK, (uint32_t)p.tpt, (uint32_t)p.T};
    rc = make_tmap_bf16(&tmA, A, 3, dims, strides, box, true);
  } else {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)T_rows};
    uint64_t strides[1] = {(uint64_t)p.K * 2};
    uint32_t box[2] = {kBK, 128};
    rc = make_tmap_bf16(&tmA, A, 2, dims, strides, box, true);
  }
  if (rc != SPK_OK) return rc;
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    uint64_t strides[1] = {(uint64_t)p.K * 2};
    uint32_t box[2] = {kBK, (uint32_t)p.wbox};
    if ((rc = make_tmap_bf16(&tmW, W, 2, dims, strides, box, true)) != SPK_OK) return rc;
  }
  return launch_gemm_maps(mode, tmA, tmW, p, st);
}

static int launch_gemm_maps(int mode, const CUtensorMap& tmA, const CUtensorMap& tmW, Params& p, cudaStream_t st) {
  // two accumulators when both fit in TMEM's 512 columns
  p.nacc = 2 * p.n_cta <= 512 ? 2 : 1;
  p.tmem_cols = tmem_cols_for(p.nacc * p.n_cta);
  // ---- stages that fit
  size_t smem = 0;
  for (p.stages = 4; p.stages >= 2; --p.stages) {
    smem = smem_layout(p, nullptr, nullptr);
    if (smem <= (size_t)kMaxSmem) break;
  }
  if (smem > (size_t)kMaxSmem) return fail(SPK_ERR_SHAPE, "tile of %d columns does not fit in shared memory", p.n_cta);

  const int sms = num_sms();
  const int total = p.num_m_tiles * p.num_n_tiles * (p.k_splits > 1 ? p.k_splits : 1);
  int clusters = sms / p.cs;
  if (clusters > total) clusters = total;
  if (clusters < 1) clusters = 1;

  void (*kern)(const CUtensorMap, const CUtensorMap, const Params);
  if (mode == MODE_TCOUPLED) kern = gemm_ln_lif_kernel<MODE_TCOUPLED>;
  else if (mode == MODE_TBCAST) kern = gemm_ln_lif_kernel<MODE_TBCAST>;
  else kern = gemm_ln_lif_kernel<MODE_PLAIN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));

  const int cfg_cs = p.cs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * p.cs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cfg_cs > 1) {
    // persistent grid: never more clusters than can be co-resident (a cluster
    // left over for a second wave would run all its tiles after the others)
    int max_clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&max_clusters, (const void*)kern, &cfg) == cudaSuccess && max_clusters > 0 &&
        max_clusters < clusters) {
      clusters = max_clusters;
      cfg.gridDim = dim3((unsigned)(clusters * cfg_cs), 1, 1);
    }
  }
  add_pdl_attr(cfg, attr);  // after the occupancy query, which describes the cluster shape alone
  e = cudaLaunchKernelEx(&cfg, kern, tmA, tmW, p);
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "gemm_ln_lif_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

// t-coupled kernel with interleaved rows (gemm_il.cu)
int launch_gemm_il(const void* A, const void* W, const float* bias, const float* gamma, const float* beta_ln,
                   float eps, const float* lif_beta, const float* lif_vth, const float* lif_vr, float gain, int T,
                   int64_t R, int K, int N, int t_broadcast, void* spk_bf16, float* spk_f32, void* residual,
                   float* ln_out, cudaStream_t st);

static bool force_generic() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SPK_GEMM_GENERIC");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

static int pick_split(int N, int* cs, int* n_cta) {
  // smallest cluster whose column slice fits one CTA's TMEM (<= 384 preferred, <= 512 allowed)
  for (int lim : {384, 512}) {
    for (int c = 1; c <= 8; ++c) {
      if (N % c) continue;
      int w = N / c;
      if (w % 32 == 0 && w <= lim) {
        *cs = c;
        *n_cta = w;
        return SPK_OK;
      }
    }
  }
  return fail(SPK_ERR_SHAPE, "LayerNorm width N=%d unsupported (needs N %% 32 == 0 and N <= 4096)", N);
}

static uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while ((int)c < n) c <<= 1;
  return c;
}

static int wbox_for(int n_cta) {
  if (n_cta <= 256) return n_cta;
  for (int b = 256; b >= 8; b -= 8)
    if (n_cta % b == 0) return b;
  return 8;
}

// Sum of the split-K partial outputs, in split order (deterministic).
__global__ void __launch_bounds__(256) sum_splits_kernel(const float4* __restrict__ part, int splits, int64_t n4,
                                                         float4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = part[i];
    for (int s = 1; s < splits; ++s) {
      const float4 b = part[(int64_t)s * n4 + i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    out[i] = a;
  }
}

// Output column tile for MN-major B operands: a multiple of 64 up to 256 that
// wastes the fewest columns (the larger one on a tie).
static int pick_nt_mn(int64_t N) {
  int best = 256;
  int64_t waste = (N + 255) / 256 * 256 - N;
  for (int w : {192, 128, 64}) {
    const int64_t ws = (N + w - 1) / w * w - N;
    if (ws < waste) {
      waste = ws;
      best = w;
    }
  }
  return best;
}

// Output column tile of the gradient GEMMs: the whole row when it fits one
// CTA's TMEM (K <= 512, a multiple of 64: the A tile is then read once per row
// block), else pick_nt_mn.
static int pick_nt_grad(int64_t K) { return (K <= 512 && K % 64 == 0) ? (int)K : pick_nt_mn(K); }

// Split count of the weight-gradient GEMM: as many splits as fill one wave of
// SMs without a second partial wave, at least 4 K blocks per split.
static int wgrad_splits(int64_t M, int64_t N, int64_t K, int* kb_per_split) {
  const int64_t nkb = (M + kBK - 1) / kBK;
  const int nt = pick_nt_grad(K);
  const int64_t tiles = ((N + 127) / 128) * ((K + nt - 1) / nt);
  int64_t splits = num_sms() / tiles;
  const int64_t most = nkb / 4 > 0 ? nkb / 4 : 1;
  if (splits > most) splits = most;
  if (splits < 1) splits = 1;
  const int64_t kbs = (nkb + splits - 1) / splits;
  *kb_per_split = (int)kbs;
  return (int)((nkb + kbs - 1) / kbs);
}

static int make_map_sw128(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                          uint32_t box_outer) {
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {inner * 2};
  uint32_t box[2] = {box_inner, box_outer};
  return make_tmap_bf16(m, base, 2, dims, strides, box, true);
}

}  // namespace spk

extern "C" {

int spk_linear_ln_lif_fwd(const void* A, const void* W, const float* bias, const float* ln_gamma,
                          const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                          const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t K, int64_t N,
                          int t_broadcast, void* spikes, int spike_dtype, void* residual, float* ln_out,
                          void* stream) {
  using namespace spk;
  SPK_REQUIRE(A && W && lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(spike_dtype == SPK_BF16 || spike_dtype == SPK_F32, SPK_ERR_INVALID, "spike dtype must be bf16 or f32");
  SPK_REQUIRE(spikes || residual, SPK_ERR_INVALID, "neither spikes nor residual output given");
  SPK_REQUIRE(T >= 1 && T <= 128 && R >= 1 && K >= 8 && K % 8 == 0 && N >= 32, SPK_ERR_SHAPE,
              "unsupported sizes T=%lld R=%lld K=%lld N=%lld (K must be a multiple of 8)", (long long)T,
              (long long)R, (long long)K, (long long)N);
  SPK_REQUIRE(R < (1ll << 31) && K < (1 << 24), SPK_ERR_SHAPE, "R or K too large");
  SPK_REQUIRE(aligned(A, 16) && aligned(W, 16), SPK_ERR_ALIGN, "A and W must be 16-byte aligned");
  SPK_REQUIRE((!spikes || aligned(spikes, 16)) && (!residual || aligned(residual, 16)), SPK_ERR_ALIGN,
              "spike / residual buffers must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Params p = {};
  if ((rc = pick_split((int)N, &p.cs, &p.n_cta)) != SPK_OK) return rc;
  p.T = (int)T;
  p.R = R;
  p.K = (int)K;
  p.N = (int)N;
  p.num_n_tiles = 1;
  p.wbox = wbox_for(p.n_cta);
  p.tmem_cols = tmem_cols_for(p.n_cta);
  p.bias = bias;
  p.gamma = ln_gamma;
  p.beta_ln = ln_beta;
  p.eps = ln_eps;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vreset;
  p.gain = in_gain;
  p.spk_bf16 = spike_dtype == SPK_BF16 ? reinterpret_cast<__nv_bfloat16*>(spikes) : nullptr;
  p.spk_f32 = spike_dtype == SPK_F32 ? reinterpret_cast<float*>(spikes) : nullptr;
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual);
  p.ln_out = ln_out;
  p.norm = 1;
  int mode;
  int64_t rows_2d = R;
  if (t_broadcast) {
    mode = MODE_TBCAST;
    p.tpt = 128;
    p.num_m_tiles = (int)((R + 127) / 128);
    if (!force_generic()) {
      rc = launch_gemm_il(A, W, bias, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vreset, in_gain, (int)T, R,
                          (int)K, (int)N, 1, p.spk_bf16, p.spk_f32, residual, ln_out,
                          reinterpret_cast<cudaStream_t>(stream));
      if (rc == SPK_OK) return check_launch("gemm_il_kernel");
      if (rc != SPK_ERR_UNSUPPORTED) return rc;
    }
  } else {
    mode = MODE_TCOUPLED;
    p.tpt = (int)(128 / T);
    p.num_m_tiles = (int)((R + p.tpt - 1) / p.tpt);
    if (!force_generic()) {
      rc = launch_gemm_il(A, W, bias, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vreset, in_gain, (int)T, R,
                          (int)K, (int)N, 0, p.spk_bf16, p.spk_f32, residual, ln_out,
                          reinterpret_cast<cudaStream_t>(stream));
      if (rc == SPK_OK) return check_launch("gemm_il_kernel");
      if (rc != SPK_ERR_UNSUPPORTED) return rc;
    }
  }
  rc = launch_gemm(mode, A, W, p, rows_2d, reinterpret_cast<cudaStream_t>(stream));
  if (rc != SPK_OK) return rc;
  return check_launch("gemm_ln_lif_kernel");
}

int spk_linear_affine_lif_fwd(const void* A, const void* W, const float* bias, const float* scale,
                              const float* shift, const float* lif_beta, const float* lif_vth,
                              const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t K, int64_t N,
                              int t_broadcast, void* spikes, int spike_dtype, void* residual, void* stream) {
  using namespace spk;
  SPK_REQUIRE(A && W && lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(spike_dtype == SPK_BF16 || spike_dtype == SPK_F32, SPK_ERR_INVALID, "spike dtype must be bf16 or f32");
  SPK_REQUIRE(spikes || residual, SPK_ERR_INVALID, "neither spikes nor residual output given");
  SPK_REQUIRE(T >= 1 && T <= 128 && R >= 1 && K >= 8 && K % 8 == 0 && N >= 32, SPK_ERR_SHAPE,
              "unsupported sizes T=%lld R=%lld K=%lld N=%lld (K must be a multiple of 8)", (long long)T,
              (long long)R, (long long)K, (long long)N);
  SPK_REQUIRE(R < (1ll << 31) && K < (1 << 24), SPK_ERR_SHAPE, "R or K too large");
  SPK_REQUIRE(aligned(A, 16) && aligned(W, 16), SPK_ERR_ALIGN, "A and W must be 16-byte aligned");
  SPK_REQUIRE((!spikes || aligned(spikes, 16)) && (!residual || aligned(residual, 16)), SPK_ERR_ALIGN,
              "spike / residual buffers must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Params p = {};
  if ((rc = pick_split((int)N, &p.cs, &p.n_cta)) != SPK_OK) return rc;
  p.T = (int)T;
  p.R = R;
  p.K = (int)K;
  p.N = (int)N;
  p.num_n_tiles = 1;
  p.wbox = wbox_for(p.n_cta);
  p.tmem_cols = tmem_cols_for(p.n_cta);
  p.bias = bias;
  p.gamma = scale;
  p.beta_ln = shift;
  p.norm = 0;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vreset;
  p.gain = in_gain;
  p.spk_bf16 = spike_dtype == SPK_BF16 ? reinterpret_cast<__nv_bfloat16*>(spikes) : nullptr;
  p.spk_f32 = spike_dtype == SPK_F32 ? reinterpret_cast<float*>(spikes) : nullptr;
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual);
  int mode;
  if (t_broadcast) {
    mode = MODE_TBCAST;
    p.tpt = 128;
    p.num_m_tiles = (int)((R + 127) / 128);
  } else {
    mode = MODE_TCOUPLED;
    p.tpt = (int)(128 / T);
    p.num_m_tiles = (int)((R + p.tpt - 1) / p.tpt);
  }
  rc = launch_gemm(mode, A, W, p, R, reinterpret_cast<cudaStream_t>(stream));
  if (rc != SPK_OK) return rc;
  return check_launch("gemm_ln_lif_kernel<affine>");
}

int spk_linear_dgrad(const void* G, const void* W, float* dX, int64_t M, int64_t N, int64_t K, void* stream) {
  using namespace spk;
  SPK_REQUIRE(G && W && dX, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(M >= 1 && N >= 8 && N % 8 == 0 && K >= 8 && K % 8 == 0 && M < (1ll << 31) && N < (1 << 24) &&
                  K < (1 << 24),
              SPK_ERR_SHAPE, "unsupported sizes M=%lld N=%lld K=%lld (N and K multiples of 8)", (long long)M,
              (long long)N, (long long)K);
  SPK_REQUIRE(aligned(G, 16) && aligned(W, 16) && aligned(dX, 16), SPK_ERR_ALIGN,
              "G, W and dX must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Params p = {};
  p.T = 1;
  p.R = M;
  p.K = (int)N;  // reduction
  p.N = (int)K;  // output columns
  p.cs = 1;
  p.n_cta = pick_nt_grad(K);
  p.num_n_tiles = (int)((K + p.n_cta - 1) / p.n_cta);
  p.num_m_tiles = (int)((M + 127) / 128);
  p.wbox = 64;
  p.tmem_cols = tmem_cols_for(p.n_cta);
  p.out_f32 = dX;
  p.vec_out = 1;
  p.b_mn = 1;
  p.k_splits = 1;
  p.tpt = 128;
  CUtensorMap tmA, tmW;
  if ((rc = make_map_sw128(&tmA, G, (uint64_t)N, (uint64_t)M, kBK, 128)) != SPK_OK) return rc;  // G [M][N]
  if ((rc = make_map_sw128(&tmW, W, (uint64_t)K, (uint64_t)N, 64, kBK)) != SPK_OK) return rc;   // W [N][K]
  rc = launch_gemm_maps(MODE_PLAIN, tmA, tmW, p, reinterpret_cast<cudaStream_t>(stream));
  if (rc != SPK_OK) return rc;
  return check_launch("gemm_ln_lif_kernel<plain, dgrad>");
}

int64_t spk_linear_wgrad_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  int kbs = 0;
  const int splits = spk::wgrad_splits(M, N, K, &kbs);
  return splits > 1 ? (int64_t)splits * N * K * (int64_t)sizeof(float) : 0;
}

int spk_linear_wgrad(const void* G, const void* X, float* dW, void* workspace, int64_t workspace_bytes, int64_t M,
                     int64_t N, int64_t K, void* stream) {
  using namespace spk;
  SPK_REQUIRE(G && X && dW, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(M >= 1 && N >= 8 && N % 8 == 0 && K >= 8 && K % 8 == 0 && M < (1ll << 31) && N < (1 << 24) &&
                  K < (1 << 24),
              SPK_ERR_SHAPE, "unsupported sizes M=%lld N=%lld K=%lld (N and K multiples of 8)", (long long)M,
              (long long)N, (long long)K);
  SPK_REQUIRE(aligned(G, 16) && aligned(X, 16) && aligned(dW, 16), SPK_ERR_ALIGN,
              "G, X and dW must be 16-byte aligned");
  const int64_t need = spk_linear_wgrad_workspace_bytes(M, N, K);
  SPK_REQUIRE(workspace_bytes >= need && (need == 0 || (workspace && aligned(workspace, 16))), SPK_ERR_INVALID,
              "workspace of %lld bytes; spk_linear_wgrad_workspace_bytes() = %lld", (long long)workspace_bytes,
              (long long)need);
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Params p = {};
  p.T = 1;
  p.R = N;       // output rows
  p.K = (int)M;  // reduction over the M rows of G and X
  p.N = (int)K;  // output columns
  p.cs = 1;
  p.n_cta = pick_nt_grad(K);
  p.num_n_tiles = (int)((K + p.n_cta - 1) / p.n_cta);
  p.num_m_tiles = (int)((N + 127) / 128);
  p.wbox = 64;
  p.tmem_cols = tmem_cols_for(p.n_cta);
  p.a_mn = 1;
  p.b_mn = 1;
  p.k_splits = wgrad_splits(M, N, K, &p.kb_per_split);
  p.split_stride = N * K;
  p.out_f32 = p.k_splits > 1 ? reinterpret_cast<float*>(workspace) : dW;
  p.vec_out = 1;
  p.tpt = 128;
  CUtensorMap tmA, tmW;
  if ((rc = make_map_sw128(&tmA, G, (uint64_t)N, (uint64_t)M, 64, kBK)) != SPK_OK) return rc;  // G [M][N]
  if ((rc = make_map_sw128(&tmW, X, (uint64_t)K, (uint64_t)M, 64, kBK)) != SPK_OK) return rc;  // X [M][K]
  rc = launch_gemm_maps(MODE_PLAIN, tmA, tmW, p, st);
  if (rc != SPK_OK) return rc;
  if ((rc = check_launch("gemm_ln_lif_kernel<plain, wgrad>")) != SPK_OK) return rc;
  if (p.k_splits > 1) {
    const int64_t n4 = N * K / 4;
    int64_t grid = (n4 + 255) / 256;
    if (grid > (int64_t)num_sms() * 8) grid = num_sms() * 8;
    sum_splits_kernel<<<(unsigned)grid, 256, 0, st>>>(reinterpret_cast<const float4*>(workspace), p.k_splits, n4,
                                                      reinterpret_cast<float4*>(dW));
    return check_launch("sum_splits_kernel");
  }
  return SPK_OK;
}

int spk_linear_fwd(const void* A, const void* W, const float* bias, float* out, int64_t M, int64_t K, int64_t N,
                   void* stream) {
  using namespace spk;
  SPK_REQUIRE(A && W && out, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(M >= 1 && K >= 8 && K % 8 == 0 && N >= 1 && M < (1ll << 31) && N < (1 << 24), SPK_ERR_SHAPE,
              "unsupported sizes M=%lld K=%lld N=%lld (K must be a multiple of 8)", (long long)M, (long long)K,
              (long long)N);
  SPK_REQUIRE(aligned(A, 16) && aligned(W, 16), SPK_ERR_ALIGN, "A and W must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Params p = {};
  p.T = 1;
  p.R = M;
  p.K = (int)K;
  p.N = (int)N;
  p.cs = 1;
  int n_pad = (int)((N + 31) / 32 * 32);
  p.n_cta = n_pad <= 256 ? n_pad : 256;
  p.num_n_tiles = (int)((N + p.n_cta - 1) / p.n_cta);
  p.num_m_tiles = (int)((M + 127) / 128);
  p.wbox = wbox_for(p.n_cta);
  p.tmem_cols = tmem_cols_for(p.n_cta);
  p.bias = bias;
  p.out_f32 = out;
  p.vec_out = (N % 4 == 0 && aligned(out, 16) && (!bias || aligned(bias, 16))) ? 1 : 0;
  p.tpt = 128;
  rc = launch_gemm(MODE_PLAIN, A, W, p, M, reinterpret_cast<cudaStream_t>(stream));
  if (rc != SPK_OK) return rc;
  return check_launch("gemm_ln_lif_kernel<plain>");
}

}  // extern "C"
