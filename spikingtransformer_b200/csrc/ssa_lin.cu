// Spiking attention without a score matrix (unmasked case), on tcgen05.
//
// Same result as the dense kernel in ssa.cu (SSA.py:145-165, :177-201,
// :234-244; plain form SSA.py:81-84) whenever no mask is applied: the
// encoder self-attention and the decoder cross-attention (Encoder.py:18,
// Decoder.py:21).  With S'[i,j] = 2 q_i.k_j + c_i - s_j + R(|i-j|),
// c_i = dh - |q_i|, s_j = |k_j|, the attention product is regrouped exactly:
//
//   O_i = sum_j S'[i,j] v_j = 2 q_i (K^T V) + c_i (1^T V) - (s^T V) + (R V)_i
//
// Every term is an integer computed exactly (bf16 operands <= 512, fp32
// accumulation < 2^24), so O equals the dense product bit for bit; the
// output stage (a = scale*O, LIF over t) is the dense kernel's.  Cost per
// (t, batch, head) is O(Nk*dh*(dh+Nq)) tensor work and O(Nq*dh) epilogue work
// instead of O(Nq*Nk) score elements.
//
// Per CTA: a persistent walk over (batch, head) items, each over its T steps;
// one unit (item, t) covers all Nq <= 256 queries (one or two 128-row blocks),
// so K and V are read once per (t, batch, head).  The log-distance matrix R
// of both query blocks (128 x Nk each, bf16, values <= 13) is built once and
// stays resident in TMEM as the A operand of the R V products.  Per unit:
//   MMA1  D1[128 x dh] = A1 V,  A1 = [K^T ; AUX^T] (MN-major, two 64-row
//         atoms: K tile and an auxiliary tile whose columns 0/1 hold 1 and
//         s_j), so D1 rows 0..dh-1 = K^T V, row 64 = 1^T V, row 65 = s^T V
//   epi   rows 0..63 of D1 -> bf16 (x2 for XNOR) B operand Mb in shared memory;
//         Mb has one extra column of ones
//   MMA2  per query block: D2 = Q [2 K^T V | 1] [+ R V]; the extra column
//         gives |q_i|, so the epilogue never reads Q
//   epi   O = D2 + (dh - |q_i|) (1^T V) - s^T V; a = scale O; LIF over t
// Warps: 0 TMA, 1 TMEM owner + MMA issuer, 2-9 epilogue (two groups of four;
// with two query blocks each group owns one, with one they split the head
// dimension).  Requirements: Nq <= 256, Nk <= 256, dh <= 64 (dh % 8 == 0).
#include "common.cuh"

namespace spk {
namespace ssal {

constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kEpi = 32 * kEpiWarps;
constexpr int kQTile = 128 * 128;   // 128 rows x 128 B
constexpr int kKVTile = 256 * 128;  // 256 rows x 128 B

struct Params {
  int T, B, H, Nq, Nk, dh;
  int QB;      // query blocks of 128 (1 or 2)
  int dsplit;  // head-dimension split between the two epilogue groups when QB = 1
  const float* scale;
  const float *lif_beta, *lif_vth, *lif_vr;
  float gain;
  __nv_bfloat16* out_bf16;
  float* out_f32;
  float* attn_out;
  int attn_tok;  // attn_out token-major [T][B][Nq][H*dh] (else [T][B][H][Nq][dh])
  int lmax, items;
  int v8;  // bf16 output rows may be written as 32-byte vectors (16-column chunks)
};

struct Smem {
  uint8_t *q, *k, *v, *aux, *mb, *rl;
  float *cs, *kv;  // 2 parities x 64
  uint64_t *q_full, *q_empty, *kv_full, *kv_empty;
  uint64_t *aux_ready, *m_full, *mb_ready, *o_full, *o_empty, *r_ready, *drain;
  uint32_t* tmem_base;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline size_t smem_layout(int lmax, uint8_t* base, Smem* s) {
  size_t off = 0;
  auto take = [&](size_t bytes, size_t al) {
    off = align_up(off, al);
    size_t o = off;
    off += bytes;
    return o;
  };
  size_t oq = take(2 * kQTile, 1024), ok = take(2 * kKVTile, 1024), ov = take(2 * kKVTile, 1024);
  size_t oaux = take(kKVTile, 1024);  // after both K slots: positive LBO from K to AUX
  size_t omb = take(2 * 64 * 128, 1024);  // two 64-column atoms: [2 K^T V | ones]
  size_t ocs = take(2 * 64 * 4, 16), okv = take(2 * 64 * 4, 16);
  size_t orl = take((size_t)lmax, 16);
  size_t ob = take(20 * 8, 8), otm = take(4, 4);
  if (s) {
    s->q = base + oq;
    s->k = base + ok;
    s->v = base + ov;
    s->aux = base + oaux;
    s->mb = base + omb;
    s->rl = base + orl;
    s->cs = reinterpret_cast<float*>(base + ocs);
    s->kv = reinterpret_cast<float*>(base + okv);
    uint64_t* b = reinterpret_cast<uint64_t*>(base + ob);
    s->q_full = b;
    s->q_empty = b + 1;
    s->kv_full = b + 2;
    s->kv_empty = b + 4;
    s->aux_ready = b + 6;
    s->m_full = b + 7;
    s->mb_ready = b + 8;
    s->o_full = b + 9;
    s->o_empty = b + 10;
    s->r_ready = b + 11;
    s->drain = b + 12;
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
  }
  return off;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int h, int row, int tb) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(0), "r"(h), "r"(row), "r"(tb)
      : "memory");
}

// DP: head width rounded up to 16; XNOR selects the S' = 2QK^T + c - s + R
// form, otherwise the plain Q K^T.  NO = DP + 16: the columns of D2 (the
// product with Mb and its ones column).
template <int DP, bool XNOR>
__global__ void __launch_bounds__(kThreads, 1)
    ssa_lin_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int NO = DP + 16;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  Smem sm;
  smem_layout(p.lmax, base, &sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  const int ksteps = (p.Nk + 15) >> 4;
  constexpr int dsteps = DP / 16;
  const int QB = p.QB;
  // per-CTA sequence of work units g = (item, t): item = blockIdx.x + k * gridDim.x
  const int n_items = p.items > (int)blockIdx.x ? (p.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int n_units = n_items * p.T;

  if (threadIdx.x == 0) {
    mbar_init(sm.q_full, 1);
    mbar_init(sm.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1 + kEpiWarps);
    }
    mbar_init(sm.aux_ready, kEpiWarps);
    mbar_init(sm.m_full, 1);
    mbar_init(sm.mb_ready, 1);
    mbar_init(sm.o_full, 1);
    mbar_init(sm.o_empty, kEpiWarps);
    mbar_init(sm.r_ready, kEpiWarps);
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  // auxiliary tile: column 0 = 1 (keys < Nk), column 1 = key sums (per step), rest 0
  for (int i = threadIdx.x; i < kKVTile / 16; i += kThreads) {
    const int r = i >> 3, c = i & 7;
    uint4 w = make_uint4(0, 0, 0, 0);
    if ((c ^ (r & 7)) == 0 && r < p.Nk) w.x = 0x3F80u;  // logical chunk 0, element 0 = 1.0
    *reinterpret_cast<uint4*>(sm.aux + i * 16) = w;
  }
  // Mb: zero, then the ones column (column DP: atom DP/64, chunk (DP%64)/8, element 0)
  for (int i = threadIdx.x; i < (2 * 64 * 128) / 16; i += kThreads) {
    const int atom = i >> 9, r = (i >> 3) & 63, c = i & 7;
    uint4 w = make_uint4(0, 0, 0, 0);
    if (atom == DP / 64 && (c ^ (r & 7)) == (DP % 64) / 8) w.x = 0x3F80u;
    *reinterpret_cast<uint4*>(sm.mb + i * 16) = w;
  }
  // log-distance table R[d] = smallest k >= 0 with (d+1) * 2^k >= L-1
  for (int d = threadIdx.x; d < p.lmax; d += kThreads) {
    const long long L1 = (long long)p.lmax - 1;
    int k = 0;
    long long x = d + 1;
    while (x < L1) {
      x <<= 1;
      ++k;
    }
    sm.rl[d] = (uint8_t)k;
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_base, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  // the setup above reads only weights and constants; activations come after this
  pdl_wait();
  // R: [0, 256) (128 columns per query block), D1: [256, 320), D2: [320, 320 + 2 NO)
  const uint32_t tm_r = tmem, tm_d1 = tmem + 256, tm_d2 = tmem + 320;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int q_ph = -1, kv_ph[2] = {-1, -1};
      for (int g = 0; g < n_units && ok; ++g) {
        const int item = (int)blockIdx.x + (g / p.T) * (int)gridDim.x, t = g % p.T;
        const int b = item / p.H, h = item % p.H;
        const int s = g & 1;
        const uint32_t ph = (uint32_t)((g >> 1) & 1);
        if (!mbar_wait(&sm.kv_empty[s], ph ^ 1u, 72)) { ok = false; break; }
        mbar_expect_tx(&sm.kv_full[s], 4 * kQTile);
        kv_ph[s] = (int)ph;
        for (int half = 0; half < 2; ++half) {
          load_4d(sm.k + s * kKVTile + half * kQTile, &tmK, &sm.kv_full[s], h, half * 128, t * p.B + b);
          load_4d(sm.v + s * kKVTile + half * kQTile, &tmV, &sm.kv_full[s], h, half * 128, t * p.B + b);
        }
        if (!mbar_wait(sm.q_empty, (uint32_t)((g & 1) ^ 1), 71)) { ok = false; break; }
        mbar_expect_tx(sm.q_full, (uint32_t)(QB * kQTile));
        q_ph = g & 1;
        for (int qb = 0; qb < QB; ++qb)
          load_4d(sm.q + qb * kQTile, &tmQ, sm.q_full, h, qb * 128, t * p.B + b);
      }
      if (!ok) {
        if (q_ph >= 0) mbar_wait(sm.q_full, (uint32_t)q_ph, 73);
        for (int i = 0; i < 2; ++i)
          if (kv_ph[i] >= 0) mbar_wait(&sm.kv_full[i], (uint32_t)kv_ph[i], 73);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    bool ok = true;
    const uint32_t id1 = idesc_bf16_f32(128, DP, 1, 1);   // A1, V: MN-major
    const uint32_t idq = idesc_bf16_f32(128, NO, 0, 1);   // Q: K-major, Mb: MN-major
    const uint32_t idr = idesc_bf16_f32(128, DP, 0, 1);   // R (TMEM), V: MN-major
    if (XNOR && n_units > 0 && !mbar_wait(sm.r_ready, 0u, 81)) ok = false;
    for (int g = 0; g < n_units && ok; ++g) {
      const int s = g & 1;
      const uint32_t ph = (uint32_t)((g >> 1) & 1);
      // MMA1: [K^T ; AUX^T] V
      if (!mbar_wait(&sm.kv_full[s], ph, 82)) { ok = false; break; }
      if (!mbar_wait(sm.aux_ready, (uint32_t)(g & 1), 83)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t ka = smem_u32(sm.k + s * kKVTile), va = smem_u32(sm.v + s * kKVTile);
        const uint32_t lbo = smem_u32(sm.aux) - ka;
        for (int kk = 0; kk < ksteps; ++kk)
          umma_bf16(tm_d1, umma_desc(ka + kk * 2048, lbo, 1024, 2), umma_desc(va + kk * 2048, kKVTile, 1024, 2),
                    id1, kk > 0 ? 1u : 0u);
        umma_commit(sm.m_full);
      }
      __syncwarp();
      // MMA2 per query block: Q [2 K^T V | 1] [+ R V]
      if (!mbar_wait(sm.mb_ready, (uint32_t)(g & 1), 84)) { ok = false; break; }
      if (!mbar_wait(sm.q_full, (uint32_t)(g & 1), 85)) { ok = false; break; }
      if (!mbar_wait(sm.o_empty, (uint32_t)((g & 1) ^ 1), 86)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t mba = smem_u32(sm.mb), va = smem_u32(sm.v + s * kKVTile);
        for (int qb = 0; qb < QB; ++qb) {
          const uint32_t qa = smem_u32(sm.q + qb * kQTile);
#pragma unroll
          for (int kk = 0; kk < dsteps; ++kk)
            umma_bf16(tm_d2 + qb * NO, umma_desc(qa + kk * 32, 16, 1024, 2), umma_desc(mba + kk * 2048, 8192, 1024, 2),
                      idq, kk > 0 ? 1u : 0u);
          if (XNOR)
            for (int kk = 0; kk < ksteps; ++kk)
              umma_bf16_ts(tm_d2 + qb * NO, tm_r + qb * 128 + kk * 8, umma_desc(va + kk * 2048, kKVTile, 1024, 2),
                           idr, 1u);
        }
        umma_commit(sm.o_full);
        umma_commit(sm.q_empty);
        umma_commit(&sm.kv_empty[s]);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) umma_commit(sm.drain);
      __syncwarp();
      mbar_wait(sm.drain, 0, 87);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;           // TMEM lane quadrant
    const int grp = ew >> 2;             // epilogue group
    const int lrow = quad * 32 + lane;   // TMEM lane = row within a 128-row block
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qb = QB == 2 ? grp : 0;    // query block of this thread's row
    const int dc0 = QB == 2 ? 0 : (grp ? p.dsplit : 0);           // first head column
    const int dcols = QB == 2 ? p.dh : (grp ? p.dh - p.dsplit : p.dsplit);
    const int qi = qb * 128 + lrow;
    const float scale = __ldg(p.scale);
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const int D = p.H * p.dh;
    bool ok = true;
    float mem[DP];
#pragma unroll
    for (int i = 0; i < DP; ++i) mem[i] = 0.0f;

    // R rows of both query blocks -> TMEM once (bf16 pairs: keys 2c and 2c+1 in column c)
    if (XNOR) {
      const int rb = QB == 2 ? grp : 0;                       // block built by this group
      const int cbeg = QB == 2 ? 0 : grp * 64, cend = QB == 2 ? 128 : cbeg + 64;
      const int ri = rb * 128 + lrow;
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        uint32_t rr[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j0 = 2 * (c0 + i), j1 = j0 + 1;
          // rows past Nq are never stored; the guard keeps their distances inside the table
          const int e0 = ri > j0 ? ri - j0 : j0 - ri, e1 = ri > j1 ? ri - j1 : j1 - ri;
          const float r0 = (j0 < p.Nk && e0 < p.lmax) ? (float)sm.rl[e0] : 0.0f;
          const float r1 = (j1 < p.Nk && e1 < p.lmax) ? (float)sm.rl[e1] : 0.0f;
          rr[i] = pack_bf16x2(r0, r1);
        }
        tmem_st32(tm_r + rb * 128 + lane_off + c0, rr);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sm.r_ready);
    }

    // key sums of unit g into the auxiliary tile; releases the K slot for reading
    auto key_sums = [&](int g) -> bool {
      const int s = g & 1;
      const uint32_t ph = (uint32_t)((g >> 1) & 1);
      if (!mbar_wait(&sm.kv_full[s], ph, 91)) return false;
      if (XNOR) {
        const int j = grp * 128 + lrow;
        const float ks = (float)row_count_sw128(sm.k + s * kKVTile, j, p.dh);
        __nv_bfloat16* slot = reinterpret_cast<__nv_bfloat16*>(sm.aux + j * 128 + ((0 ^ (j & 7)) << 4)) + 1;
        *slot = __float2bfloat16_rn(ks);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(sm.aux_ready);
        mbar_arrive(&sm.kv_empty[s]);
      }
      return true;
    };

    // A: K^T V of unit g -> bf16 operand (x2 for XNOR); 1^T V, s^T V -> shared floats (parity g & 1)
    auto build_mb = [&](int g) -> bool {
      const int par = g & 1;
      if (!mbar_wait(sm.m_full, (uint32_t)(g & 1), 93)) return false;
      tc_fence_after();
      if (grp == 0 && quad < 3) {
        const float f = XNOR ? 2.0f : 1.0f;
#pragma unroll
        for (int c0 = 0; c0 < DP; c0 += 16) {
          float d1[16];
          tmem_ld16(tm_d1 + lane_off + c0, d1);
          if (quad < 2) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint4 w;
              w.x = pack_bf16x2(f * d1[8 * c + 0], f * d1[8 * c + 1]);
              w.y = pack_bf16x2(f * d1[8 * c + 2], f * d1[8 * c + 3]);
              w.z = pack_bf16x2(f * d1[8 * c + 4], f * d1[8 * c + 5]);
              w.w = pack_bf16x2(f * d1[8 * c + 6], f * d1[8 * c + 7]);
              const int ch = c0 / 8 + c;
              *reinterpret_cast<uint4*>(sm.mb + lrow * 128 + ((ch ^ (lrow & 7)) << 4)) = w;
            }
          } else if (XNOR && lane < 2) {
            float* dst = (lane == 0 ? sm.cs : sm.kv) + par * 64 + c0;
#pragma unroll
            for (int c = 0; c < 16; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(d1[c], d1[c + 1], d1[c + 2], d1[c + 3]);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1, kEpi);
      if (threadIdx.x == 64) mbar_arrive(sm.mb_ready);
      return true;
    };

    // Unit order with EARLY (head width <= 48): the operand of unit g+1 is built as soon as unit
    // g's product has been read out of TMEM, so the product of unit g+1 runs on the tensor cores
    // while unit g's output is computed; key sums run two units ahead.  Wider heads keep the
    // product in TMEM while the output is computed (the registers hold the LIF state).
    constexpr bool EARLY = DP <= 48;
    constexpr int NCH = DP / 16;
    auto in_range = [&](int c) { return !(c * 16 + 16 <= dc0 || c * 16 >= dc0 + dcols); };
    if (n_units > 0) ok = key_sums(0);
    if (EARLY) {
      if (ok && n_units > 0) ok = build_mb(0);
      if (ok && n_units > 1) ok = key_sums(1);
    }
    // unit position (step t, batch b, head h), advanced one unit at a time
    // with one division per item
    int t = 0, item = (int)blockIdx.x, b = item / p.H, h = item - b * p.H;
    for (int g = 0; g < n_units && ok; ++g) {
      if (g > 0 && ++t == p.T) {
        t = 0;
        item += (int)gridDim.x;
        b = item / p.H;
        h = item - b * p.H;
      }
      const int par = g & 1;
      if (t == 0) {
#pragma unroll
        for (int i = 0; i < DP; ++i) mem[i] = 0.0f;
      }
      if (!EARLY) {
        if (!build_mb(g)) { ok = false; break; }
        if (g + 1 < n_units && !key_sums(g + 1)) { ok = false; break; }
      }
      if (!mbar_wait(sm.o_full, (uint32_t)(g & 1), 94)) { ok = false; break; }
      tc_fence_after();
      const uint32_t ta = tm_d2 + qb * NO + lane_off;
      const int64_t obase = (((int64_t)t * p.B + b) * p.Nq + qi) * D + (int64_t)h * p.dh;
      float* aout = !p.attn_out ? nullptr
                    : p.attn_tok ? p.attn_out + obase
                                 : p.attn_out + ((((int64_t)t * p.B + b) * p.H + h) * p.Nq + qi) * p.dh;
      const float* csp = sm.cs + par * 64;
      const float* kvp = sm.kv + par * 64;
      const bool row_ok = qi < p.Nq;
      uint32_t rq = 0;
      if (XNOR) {
        tmem_ld1_raw(ta + DP, rq);  // the ones column: |q_i|
        tmem_wait_ld();
        asm volatile("" : "+r"(rq) : : "memory");
      }
      const float c_row = XNOR ? (float)p.dh - __uint_as_float(rq) : 0.0f;
      const float2 c2 = make_float2(c_row, c_row), scale2 = make_float2(scale, scale);
      const float2 gain2 = make_float2(p.gain, p.gain), beta2 = make_float2(beta, beta);
      // O = D2 + (dh - |q_i|) (1^T V) - s^T V, a = scale O, LIF over t, spikes, for the 16 columns
      // of chunk c.  Packed fp32x2 arithmetic; every product and sum rounds as the scalar
      // reference (the integer terms are exact in any order).
      auto out_chunk = [&](int c, const uint32_t (&rc)[16]) {
        const int c0 = c * 16;
        uint32_t bits[8];  // bf16 spike pairs of the chunk's 16 columns
#pragma unroll
        for (int d8 = 0; d8 < 16; d8 += 8) {
          const int d0 = c0 + d8;
          if (d0 < dc0 || d0 >= dc0 + dcols) continue;
#pragma unroll
          for (int i = 0; i < 8; i += 4) {
            const float4 cs4 = *reinterpret_cast<const float4*>(csp + d0 + i);
            const float4 kv4 = *reinterpret_cast<const float4*>(kvp + d0 + i);
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
              const uint32_t* r = rc + d8 + i + j;
              float2 ov = make_float2(__uint_as_float(r[0]), __uint_as_float(r[1]));
              if (XNOR) {
                const float2 cs2 = j == 0 ? make_float2(cs4.x, cs4.y) : make_float2(cs4.z, cs4.w);
                const float2 kv2 = j == 0 ? make_float2(kv4.x, kv4.y) : make_float2(kv4.z, kv4.w);
                ov = add2(fma2(c2, cs2, ov), make_float2(-kv2.x, -kv2.y));
              }
              const float2 a = mul2(ov, scale2);
              const int dd = d0 + i + j;
              if (aout) *reinterpret_cast<float2*>(aout + dd) = a;
              const float2 cu = mul2(a, gain2);  // exact when the gain is 1
              const float2 u = add2(mul2(make_float2(mem[dd], mem[dd + 1]), beta2), cu);
              const bool f0 = u.x > vth, f1 = u.y > vth;
              mem[dd] = f0 ? vr : u.x;
              mem[dd + 1] = f1 ? vr : u.y;
              bits[(d8 + i + j) >> 1] = (f0 ? 0x3F80u : 0u) | (f1 ? 0x3F800000u : 0u);
            }
          }
        }
        const bool whole = c0 >= dc0 && c0 + 16 <= dc0 + dcols;
        if (p.out_bf16 && whole && p.v8) {
          // the chunk's 32 bytes in one store: whole sectors
          st_global_v8(p.out_bf16 + obase + c0, make_uint4(bits[0], bits[1], bits[2], bits[3]),
                       make_uint4(bits[4], bits[5], bits[6], bits[7]));
        } else if (p.out_bf16) {
#pragma unroll
          for (int d8 = 0; d8 < 16; d8 += 8) {
            const int d0 = c0 + d8;
            if (d0 < dc0 || d0 >= dc0 + dcols) continue;
            const int w = d8 >> 1;
            *reinterpret_cast<uint4*>(p.out_bf16 + obase + d0) = make_uint4(bits[w], bits[w + 1], bits[w + 2], bits[w + 3]);
          }
        }
        if (p.out_f32) {
#pragma unroll
          for (int d8 = 0; d8 < 16; d8 += 8) {
            const int d0 = c0 + d8;
            if (d0 < dc0 || d0 >= dc0 + dcols) continue;
            const uint32_t* bw = bits + (d8 >> 1);
            float4 lo, hi;
            lo.x = (bw[0] & 0xFFFFu) ? 1.0f : 0.0f; lo.y = (bw[0] >> 16) ? 1.0f : 0.0f;
            lo.z = (bw[1] & 0xFFFFu) ? 1.0f : 0.0f; lo.w = (bw[1] >> 16) ? 1.0f : 0.0f;
            hi.x = (bw[2] & 0xFFFFu) ? 1.0f : 0.0f; hi.y = (bw[2] >> 16) ? 1.0f : 0.0f;
            hi.z = (bw[3] & 0xFFFFu) ? 1.0f : 0.0f; hi.w = (bw[3] >> 16) ? 1.0f : 0.0f;
            *reinterpret_cast<float4*>(p.out_f32 + obase + d0) = lo;
            *reinterpret_cast<float4*>(p.out_f32 + obase + d0 + 4) = hi;
          }
        }
      };
      if constexpr (EARLY) {
        // all of D2 into registers, the accumulator back to the MMA warp, the next operand
        uint32_t dreg[NCH][16];
#pragma unroll
        for (int c = 0; c < NCH; ++c)
          if (in_range(c)) tmem_ld16_raw(ta + c * 16, dreg[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < NCH; ++c) reg_fence16(dreg[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.o_empty);
        if (g + 1 < n_units && !build_mb(g + 1)) { ok = false; break; }
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < NCH; ++c)
            if (in_range(c)) out_chunk(c, dreg[c]);
        }
        if (g + 2 < n_units && !key_sums(g + 2)) { ok = false; break; }
      } else {
        // chunk by chunk (16 columns), then the accumulator back to the MMA warp
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          if (!in_range(c)) continue;
          uint32_t rbuf[16];
          tmem_ld16_raw(ta + c * 16, rbuf);
          tmem_wait_ld_fence(rbuf);
          if (row_ok) out_chunk(c, rbuf);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.o_empty);
      }
    }
    (void)ok;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace ssal

SPK_DEFINE_ERROR_READER(ssa_lin_read_device_error)

// Host launcher used by spk_ssa_fwd for unmasked attention; returns
// SPK_ERR_UNSUPPORTED when the sizes are outside this kernel's range.
int launch_ssa_lin(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, int T, int B, int H,
                   int Nq, int Nk, int dh, int variant, const float* scale, const float* lif_beta,
                   const float* lif_vth, const float* lif_vr, float gain, void* out_bf16, float* out_f32,
                   float* attn_out, bool attn_token_major, cudaStream_t st) {
  using namespace ssal;
  if (Nq > 256 || Nk > 256 || dh > 64 || dh % 8 != 0) return SPK_ERR_UNSUPPORTED;
  Params p = {};
  p.T = T;
  p.B = B;
  p.H = H;
  p.Nq = Nq;
  p.Nk = Nk;
  p.dh = dh;
  p.scale = scale;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vr;
  p.gain = gain;
  p.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  p.v8 = dh % 16 == 0 && aligned(out_bf16, 32);
  p.out_f32 = out_f32;
  p.attn_out = attn_out;
  p.attn_tok = attn_token_major ? 1 : 0;
  p.QB = (Nq + 127) / 128;
  p.dsplit = ((dh / 8 + 1) / 2) * 8;
  p.lmax = Nq > Nk ? Nq : Nk;
  const long long items = (long long)B * H;
  if (items >= (1ll << 31)) return fail(SPK_ERR_SHAPE, "too many attention work items");
  p.items = (int)items;
  const int dp = (dh + 15) / 16 * 16;
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const Params);
  const bool x = variant == 1;
  switch (dp) {
    case 16: kern = x ? ssa_lin_kernel<16, true> : ssa_lin_kernel<16, false>; break;
    case 32: kern = x ? ssa_lin_kernel<32, true> : ssa_lin_kernel<32, false>; break;
    case 48: kern = x ? ssa_lin_kernel<48, true> : ssa_lin_kernel<48, false>; break;
    default: kern = x ? ssa_lin_kernel<64, true> : ssa_lin_kernel<64, false>; break;
  }
  size_t smem = smem_layout(p.lmax, nullptr, nullptr);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  int grid = num_sms();
  if (grid > p.items) grid = p.items;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  add_pdl_attr(cfg, attr);
  e = cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, p);
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "ssa_lin_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

}  // namespace spk
