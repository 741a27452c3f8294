// Spiking attention for short sequences (Nq, Nk <= 64), any mask, on tcgen05.
//
// Same contract and arithmetic as the dense kernel in ssa.cu (flofiz/
// SpikingTransformer SSA.py:145-165 XNOR scores, :177-201 log-distance bias,
// :234-244 +bias, *mask, (*scale) @ V, LIF; plain form SSA.py:81-86).  The
// decoder's masked self-attention (Nq = Nk = 64, Decoder.py:18) fills only
// half of a 128-row tensor-core tile, so this kernel packs two (batch, head)
// pairs ("slots") into every tile: rows 0-63 hold slot 0's queries and keys,
// rows 64-127 slot 1's.
//
//   S = Q K^T   one 128 x 128 tcgen05.mma (fp32 in TMEM; integer counts, exact)
//   P           the epilogue writes only the two diagonal 64 x 64 blocks
//               (XNOR transform, bias, mask, bf16 integers); the off-diagonal
//               blocks are zeroed once and never written, so P V mixes no
//               values across slots
//   O = P V     tcgen05.mma with V as an MN-major operand (exact integer sums)
//   a = scale O, LIF over t in registers, bf16 / fp32 spikes
//
// CTAs are persistent over items (slot pairs); a CTA walks its items' T steps
// as a sequence of units.  Q, K, V, S, P and O are double-buffered, and the
// epilogue is software-pipelined: in iteration g it builds P of unit g, then
// emits the spikes of unit g-1, whose P V product ran meanwhile.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2-9 epilogue.  Epilogue
// warp w reads TMEM lane quadrant w % 4; warps 2-5 own key columns 0-31 of
// their slot and the first half of the head dimension, warps 6-9 key columns
// 32-63 and the second half.  Every wait is bounded (see common.cuh).

#include "common.cuh"

namespace spk {
namespace sssk {

constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kTile = 128 * 128;  // 128 rows x 128 bytes (64 bf16)
constexpr int kHalf = 64 * 128;   // one slot's 64 rows
constexpr int kMaxLen = 64;

struct Params {
  int T, B, H, Nq, Nk, dh, dsplit;
  int mode;       // 0 plain, 1 xnor
  int mask_mode;  // 0 none, 1 causal (key <= query), 2 dense u8
  int mask_vec;   // dense mask rows may be read as 16-byte vectors
  const uint8_t* mask;
  int64_t m_st, m_sb, m_sh, m_sq;  // element strides of the dense mask (key stride 1)
  const float* scale;
  const float* lif_beta;
  const float* lif_vth;
  const float* lif_vr;
  float gain;
  __nv_bfloat16* out_bf16;  // [T][B][Nq][H*dh]
  float* out_f32;
  float* attn_out;          // optional [T][B][H][Nq][dh] (LIF input)
  int items;                // ceil(B*H / 2)
  int lmax;                 // max(Nq, Nk)
};

struct Smem {
  uint8_t* q;   // 2 x kTile
  uint8_t* k;   // 2 x kTile
  uint8_t* v;   // 2 x kTile
  uint8_t* p;   // 2 x (2 x kTile): 128 rows x 128 keys bf16 = two 64-key atoms
  float* ks;    // 2 x 128 key sums
  float* cq;    // 2 x 128 dh - query sums
  uint8_t* rl;  // log-distance table [kMaxLen]
  uint64_t *full, *empty, *sums, *s_full, *s_empty, *p_full, *p_empty, *o_full, *o_empty, *drain;
  uint32_t* tmem_base;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline size_t smem_layout(uint8_t* base, Smem* s) {
  size_t off = 0;
  auto take = [&](size_t bytes, size_t al) {
    off = align_up(off, al);
    size_t o = off;
    off += bytes;
    return o;
  };
  size_t oq = take(2 * kTile, 1024), ok = take(2 * kTile, 1024), ov = take(2 * kTile, 1024);
  size_t op = take(4 * kTile, 1024);
  size_t oks = take(2 * 128 * 4, 16), ocq = take(2 * 128 * 4, 16);
  size_t orl = take(kMaxLen, 16);
  size_t ob = take(19 * 8, 8);
  size_t otm = take(4, 4);
  if (s) {
    s->q = base + oq;
    s->k = base + ok;
    s->v = base + ov;
    s->p = base + op;
    s->ks = reinterpret_cast<float*>(base + oks);
    s->cq = reinterpret_cast<float*>(base + ocq);
    s->rl = base + orl;
    uint64_t* b = reinterpret_cast<uint64_t*>(base + ob);
    s->full = b + 0;
    s->empty = b + 2;
    s->sums = b + 4;
    s->s_full = b + 6;
    s->s_empty = b + 8;
    s->p_full = b + 10;
    s->p_empty = b + 12;
    s->o_full = b + 14;
    s->o_empty = b + 16;
    s->drain = b + 18;
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
  }
  return off;
}

// sum of the bf16 {0,1} values of row r of a 128B-swizzled tile (first n elems)
__device__ __forceinline__ float row_sum_sw128(const uint8_t* tile, int r, int n) {
  float s = 0.0f;
  const int chunks = (n + 7) >> 3;
  for (int c = 0; c < chunks; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(tile + r * 128 + ((c ^ (r & 7)) << 4));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      s += f.x + f.y;
    }
  }
  return s;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    ssa_short_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem sm;
  smem_layout(smem_raw, &sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  const int BH = p.B * p.H;
  const int my_items = (p.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int G = my_items * p.T;  // units of this CTA
  const int dsteps = (p.dh + 15) >> 4;

  // zero every operand buffer once: the off-diagonal blocks of P stay zero for
  // the whole kernel, and an unused slot of the last item reads finite data
  {
    uint4 z = make_uint4(0u, 0u, 0u, 0u);
    uint4* b = reinterpret_cast<uint4*>(sm.q);
    const int n = (10 * kTile) / 16;  // q, k, v (2 each) and p (4) are contiguous
    for (int i = threadIdx.x; i < n; i += kThreads) b[i] = z;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1 + kEpiWarps);
      mbar_init(&sm.sums[i], kEpiWarps);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], kEpiWarps);
      mbar_init(&sm.p_full[i], kEpiWarps);
      mbar_init(&sm.p_empty[i], 1);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], kEpiWarps);
    }
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_base, 512);
    tmem_relinquish();
  }
  // log-distance bias table R[d] = smallest k >= 0 with (d+1) * 2^k >= L-1
  for (int d = threadIdx.x; d < kMaxLen; d += kThreads) {
    const int L1 = p.lmax - 1;
    int k = 0, x = d + 1;
    while (x < L1) {
      x <<= 1;
      ++k;
    }
    sm.rl[d] = (uint8_t)k;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  // the setup above reads only weights and constants; activations come after this
  pdl_wait();
  const uint32_t tm_s = tmem, tm_o = tmem + 256;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int last_ph[2] = {-1, -1};
      for (int g = 0; g < G; ++g) {
        const int s = g & 1;
        if (!mbar_wait(&sm.empty[s], ((g >> 1) & 1) ^ 1u, 141)) { ok = false; break; }
        const int item = (int)blockIdx.x + (g / p.T) * (int)gridDim.x, t = g % p.T;
        const int nslots = (2 * item + 1 < BH) ? 2 : 1;
        mbar_expect_tx(&sm.full[s], (uint32_t)(3 * nslots * kHalf));
        last_ph[s] = (g >> 1) & 1;
        for (int sl = 0; sl < nslots; ++sl) {
          const int bh = 2 * item + sl, b = bh / p.H, h = bh % p.H, z = t * p.B + b;
          // 4-D maps {dh, H, N, T*B}, box {64, 1, 64, 1}: d >= dh and rows >= N read as zero
          tma_load_4d(sm.q + s * kTile + sl * kHalf, &tmQ, &sm.full[s], 0, h, 0, z);
          tma_load_4d(sm.k + s * kTile + sl * kHalf, &tmK, &sm.full[s], 0, h, 0, z);
          tma_load_4d(sm.v + s * kTile + sl * kHalf, &tmV, &sm.full[s], 0, h, 0, z);
        }
      }
      if (!ok) {
        for (int i = 0; i < 2; ++i)
          if (last_ph[i] >= 0) mbar_wait(&sm.full[i], (uint32_t)last_ph[i], 142);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    bool ok = true;
    const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
    const uint32_t idesc_pv = idesc_bf16_f32(128, dsteps * 16, 0, 1);
    auto issue_s = [&](int g) -> bool {
      const int s = g & 1;
      if (!mbar_wait(&sm.full[s], (g >> 1) & 1, 151)) return false;
      if (!mbar_wait(&sm.s_empty[s], ((g >> 1) & 1) ^ 1u, 152)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sm.q + s * kTile), ka = smem_u32(sm.k + s * kTile);
        for (int kk = 0; kk < dsteps; ++kk)
          umma_bf16(tm_s + s * 128, umma_desc(qa + kk * 32, 16, 1024, 2), umma_desc(ka + kk * 32, 16, 1024, 2),
                    idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&sm.s_full[s]);
      }
      __syncwarp();
      return true;
    };
    if (G > 0 && !issue_s(0)) ok = false;
    for (int g = 0; g < G && ok; ++g) {
      if (g + 1 < G && !issue_s(g + 1)) { ok = false; break; }
      const int s = g & 1;
      if (!mbar_wait(&sm.p_full[s], (g >> 1) & 1, 153)) { ok = false; break; }
      if (!mbar_wait(&sm.o_empty[s], ((g >> 1) & 1) ^ 1u, 154)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_u32(sm.p + s * 2 * kTile), va = smem_u32(sm.v + s * kTile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t adesc = umma_desc(pa + (kk >> 2) * kTile + (kk & 3) * 32, 16, 1024, 2);
          const uint64_t bdesc = umma_desc(va + kk * 2048, kTile, 1024, 2);
          umma_bf16(tm_o + s * 64, adesc, bdesc, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.o_full[s]);
        umma_commit(&sm.p_empty[s]);
        umma_commit(&sm.empty[s]);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) umma_commit(sm.drain);
      __syncwarp();
      mbar_wait(sm.drain, 0, 155);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int quad = warp & 3, half = ew >> 2;
    const int row = quad * 32 + lane;  // tile row
    const int slot = row >> 6, qi = row & 63;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float scale = __ldg(p.scale);
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const int D = p.H * p.dh;
    const int dcol0 = half ? p.dsplit : 0;
    const int dcols = half ? p.dh - p.dsplit : p.dsplit;
    const int kc0 = half * 32;  // first key (within the slot) of this warp's columns
    float mem[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) mem[i] = 0.0f;
    // dense masks read as 16-byte vectors are loaded one unit ahead (the 32
    // mask bytes of this thread's row and key columns), so their latency
    // hides behind the previous unit's work
    // the log-distance bias of this thread's row and 32 key columns: the same for
    // every unit, so it stays in registers (XNOR form only)
    float rbias[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int kj = kc0 + i;
      const int dist = qi > kj ? qi - kj : kj - qi;
      rbias[i] = (p.mode == 1 && dist < p.lmax) ? (float)sm.rl[dist] : 0.0f;
    }
    const bool mask_pf = p.mask_mode == 2 && p.mask_vec && kc0 + 32 <= p.Nk;
    auto mask_load = [&](int gg, uint4& m0, uint4& m1) {
      const int it = (int)blockIdx.x + (gg / p.T) * (int)gridDim.x, tt = gg % p.T;
      const int bhh = 2 * it + slot;
      m0 = make_uint4(0u, 0u, 0u, 0u);
      m1 = m0;
      if (bhh < BH && qi < p.Nq) {
        const int b = bhh / p.H, h = bhh % p.H;
        const uint4* mrow = reinterpret_cast<const uint4*>(p.mask + tt * p.m_st + b * p.m_sb + h * p.m_sh +
                                                           (int64_t)qi * p.m_sq + kc0);
        m0 = __ldg(mrow);
        m1 = __ldg(mrow + 1);
      }
    };
    uint4 pm0 = make_uint4(0u, 0u, 0u, 0u), pm1 = pm0;
    if (mask_pf && G > 0) mask_load(0, pm0, pm1);
    bool ok = true;
    for (int g = 0; g <= G && ok; ++g) {
      if (g < G) {
        // ---- build P of unit g
        const int s = g & 1;
        const int item = (int)blockIdx.x + (g / p.T) * (int)gridDim.x, t = g % p.T;
        const int bh = 2 * item + slot;
        uint32_t pf_bits = 0u;
        if (mask_pf) {
          const uint32_t w[8] = {pm0.x, pm0.y, pm0.z, pm0.w, pm1.x, pm1.y, pm1.z, pm1.w};
#pragma unroll
          for (int i = 0; i < 32; ++i) pf_bits |= (((w[i >> 2] >> ((i & 3) * 8)) & 0xffu) != 0u ? 1u : 0u) << i;
          if (g + 1 < G) mask_load(g + 1, pm0, pm1);
        }
        if (!mbar_wait(&sm.full[s], (g >> 1) & 1, 161)) { ok = false; break; }
        if (p.mode == 1) {
          if (half == 0)
            sm.ks[s * 128 + row] = row_sum_sw128(sm.k + s * kTile, row, p.dh);
          else
            sm.cq[s * 128 + row] = (float)p.dh - row_sum_sw128(sm.q + s * kTile, row, p.dh);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.empty[s]);
          if (p.mode == 1) mbar_arrive(&sm.sums[s]);
        }
        if (p.mode == 1 && !mbar_wait(&sm.sums[s], (g >> 1) & 1, 162)) { ok = false; break; }
        if (!mbar_wait(&sm.s_full[s], (g >> 1) & 1, 163)) { ok = false; break; }
        if (!mbar_wait(&sm.p_empty[s], ((g >> 1) & 1) ^ 1u, 164)) { ok = false; break; }
        tc_fence_after();
        uint32_t raw[32];
        tmem_ld32_raw(tm_s + s * 128 + lane_off + slot * 64 + kc0, raw);
        const float c_row = p.mode == 1 ? sm.cq[s * 128 + row] : 0.0f;
        const float* ks = sm.ks + s * 128 + slot * 64;
        uint32_t mbits = 0xffffffffu;  // keep bit per key column of this warp
        if (mask_pf) {
          mbits = pf_bits;
        } else if (p.mask_mode == 2) {
          mbits = 0u;
          if (bh < BH && qi < p.Nq) {
            const int b = bh / p.H, h = bh % p.H;
            const uint8_t* mrow = p.mask + t * p.m_st + b * p.m_sb + h * p.m_sh + (int64_t)qi * p.m_sq + kc0;
            if (p.mask_vec && kc0 + 32 <= p.Nk) {
              const uint4 m0 = __ldg(reinterpret_cast<const uint4*>(mrow));
              const uint4 m1 = __ldg(reinterpret_cast<const uint4*>(mrow) + 1);
              const uint32_t w[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
              for (int i = 0; i < 32; ++i) mbits |= (((w[i >> 2] >> ((i & 3) * 8)) & 0xffu) != 0u ? 1u : 0u) << i;
            } else {
              for (int i = 0; i < 32 && kc0 + i < p.Nk; ++i) mbits |= (mrow[i] != 0 ? 1u : 0u) << i;
            }
          }
        } else if (p.mask_mode == 1) {
          // key kj = kc0 + i is kept when kj <= qi
          const int n = qi - kc0 + 1;
          mbits = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
        }
        if (p.Nk - kc0 < 32) {
          const int n = p.Nk - kc0;
          mbits &= n <= 0 ? 0u : ((1u << n) - 1u);
        }
        tmem_wait_ld_fence32(raw);
        float v[32];
#pragma unroll
        for (int i0 = 0; i0 < 32; i0 += 4) {
          // four key sums in one 16-byte load (the same address in every lane)
          const float4 k4 = p.mode == 1 ? *reinterpret_cast<const float4*>(ks + kc0 + i0)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + u;
            float sc = __uint_as_float(raw[i]);
            if (p.mode == 1) sc = fmaf(2.0f, sc, c_row - kv[u]) + rbias[i];
            v[i] = ((mbits >> i) & 1u) ? sc : 0.0f;
          }
        }
        // 32 keys of row `row` into the slot's 64-key atom (K-major, 128-byte swizzle)
        uint8_t* prow = sm.p + s * 2 * kTile + slot * kTile + row * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int ch = half * 4 + c;
          uint4 w;
          w.x = pack_bf16x2(v[c * 8 + 0], v[c * 8 + 1]);
          w.y = pack_bf16x2(v[c * 8 + 2], v[c * 8 + 3]);
          w.z = pack_bf16x2(v[c * 8 + 4], v[c * 8 + 5]);
          w.w = pack_bf16x2(v[c * 8 + 6], v[c * 8 + 7]);
          *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) = w;
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.s_empty[s]);
          mbar_arrive(&sm.p_full[s]);
        }
      }
      if (g >= 1) {
        // ---- spikes of unit u = g - 1
        const int u = g - 1, s = u & 1;
        const int item = (int)blockIdx.x + (u / p.T) * (int)gridDim.x, t = u % p.T;
        const int bh = 2 * item + slot;
        if (!mbar_wait(&sm.o_full[s], (u >> 1) & 1, 165)) { ok = false; break; }
        tc_fence_after();
        uint32_t raw[32];
        tmem_ld32_raw(tm_o + s * 64 + lane_off + dcol0, raw);
        tmem_wait_ld_fence32(raw);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_empty[s]);
        if (t == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mem[i] = 0.0f;
        }
        if (bh < BH && qi < p.Nq) {
          const int b = bh / p.H, h = bh % p.H;
          const int64_t obase = (((int64_t)t * p.B + b) * p.Nq + qi) * D + (int64_t)h * p.dh + dcol0;
          float* aout = p.attn_out
                            ? p.attn_out + ((((int64_t)t * p.B + b) * p.H + h) * p.Nq + qi) * p.dh + dcol0
                            : nullptr;
#pragma unroll
          for (int d0 = 0; d0 < 32; d0 += 8) {
            if (d0 < dcols) {
              float sp[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float a = __fmul_rn(__uint_as_float(raw[d0 + i]), scale);
                if (aout) aout[d0 + i] = a;
                const float cur = p.gain != 1.0f ? __fmul_rn(a, p.gain) : a;
                const float uu = __fadd_rn(__fmul_rn(mem[d0 + i], beta), cur);
                const bool fire = uu > vth;
                sp[i] = fire ? 1.0f : 0.0f;
                mem[d0 + i] = fire ? vr : uu;
              }
              if (p.out_bf16) {
                uint4 w;
                w.x = pack_bf16x2(sp[0], sp[1]);
                w.y = pack_bf16x2(sp[2], sp[3]);
                w.z = pack_bf16x2(sp[4], sp[5]);
                w.w = pack_bf16x2(sp[6], sp[7]);
                *reinterpret_cast<uint4*>(p.out_bf16 + obase + d0) = w;
              }
              if (p.out_f32) {
                *reinterpret_cast<float4*>(p.out_f32 + obase + d0) = make_float4(sp[0], sp[1], sp[2], sp[3]);
                *reinterpret_cast<float4*>(p.out_f32 + obase + d0 + 4) = make_float4(sp[4], sp[5], sp[6], sp[7]);
              }
            }
          }
        }
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

}  // namespace sssk

SPK_DEFINE_ERROR_READER(ssa_short_read_device_error)

static int make_map64(CUtensorMap* m, const void* ptr, int dh, int H, int N, int TB) {
  uint64_t dims[4] = {(uint64_t)dh, (uint64_t)H, (uint64_t)N, (uint64_t)TB};
  uint64_t strides[3] = {(uint64_t)dh * 2, (uint64_t)H * dh * 2, (uint64_t)N * H * dh * 2};
  uint32_t box[4] = {64, 1, 64, 1};
  return make_tmap_bf16(m, ptr, 4, dims, strides, box, true);
}

// Returns SPK_ERR_UNSUPPORTED (nothing launched) for shapes it does not take.
int launch_ssa_short(const void* q, const void* k, const void* v, int T, int B, int H, int Nq, int Nk, int dh,
                     int variant, int mask_mode, const uint8_t* mask, int64_t m_st, int64_t m_sb, int64_t m_sh,
                     int64_t m_sq, const float* scale, const float* lif_beta, const float* lif_vth,
                     const float* lif_vr, float gain, void* out_bf16, float* out_f32, float* attn_out,
                     cudaStream_t st) {
  using namespace sssk;
  if (Nq > kMaxLen || Nk > kMaxLen || dh > 64 || dh % 8 != 0) return SPK_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_map64(&tq, q, dh, H, Nq, T * B)) != SPK_OK) return rc;
  if ((rc = make_map64(&tk, k, dh, H, Nk, T * B)) != SPK_OK) return rc;
  if ((rc = make_map64(&tv, v, dh, H, Nk, T * B)) != SPK_OK) return rc;
  Params p = {};
  p.T = T;
  p.B = B;
  p.H = H;
  p.Nq = Nq;
  p.Nk = Nk;
  p.dh = dh;
  p.dsplit = ((dh / 8 + 1) / 2) * 8;
  p.mode = variant;
  p.mask_mode = mask_mode;
  p.mask = mask;
  p.m_st = m_st;
  p.m_sb = m_sb;
  p.m_sh = m_sh;
  p.m_sq = m_sq;
  p.mask_vec = mask_mode == 2 && aligned(mask, 16) && m_st % 16 == 0 && m_sb % 16 == 0 && m_sh % 16 == 0 &&
               m_sq % 16 == 0;
  p.scale = scale;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vr;
  p.gain = gain;
  p.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  p.out_f32 = out_f32;
  p.attn_out = attn_out;
  p.items = (B * H + 1) / 2;
  p.lmax = Nq > Nk ? Nq : Nk;
  const size_t smem = smem_layout(nullptr, nullptr) + 1024;
  cudaError_t e = cudaFuncSetAttribute(ssa_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
  e = cudaLaunchKernelEx(&cfg, ssa_short_kernel, tq, tk, tv, p);
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "ssa_short_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

}  // namespace spk
