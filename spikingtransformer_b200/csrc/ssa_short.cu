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
//   S = Q K^T   one 128 x 128 tcgen05.mma (fp32 in TMEM; integer counts, exact);
//               row r of slot sl reads its own keys at columns 64 sl .. 64 sl + 63
//   P           128 rows x 64 keys: each row holds its own slot's keys (XNOR
//               transform, bias, mask, bf16 integers)
//   O = P [V0 | V1]  K = 64, N = 128, with V as an MN-major operand whose two
//               64-column atoms are the two slots' V tiles (exact integer
//               sums); slot sl's rows keep columns 64 sl .. 64 sl + dh - 1.
//               Half of the product is discarded, but a one-CTA M = 128 MMA
//               costs about the same at N = 128 as at N = 48, so four N = 128
//               instructions replace eight block-diagonal N = 48 ones
//   a = scale O, LIF over t in registers, bf16 / fp32 spikes
//
// CTAs are persistent over items (slot pairs); a CTA walks its items' T steps
// as a sequence of units.  Q, K and V sit in a ring of three stages, so the
// loads of the next two units are in flight while a unit is computed (a unit
// moves about 37 KB, and one SM's share of HBM needs about two units in
// flight to cover the load latency); S, P and O are double-buffered.  The
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
constexpr int kStages = 3;  // Q/K/V ring

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
  uint8_t* q;   // kStages x kTile
  uint8_t* k;   // kStages x kTile
  uint8_t* v;   // kStages x kTile
  uint8_t* p;   // 2 x kTile: 128 rows x 64 keys bf16 (one 64-key atom)
  float* ks;    // kStages x 128 key sums
  float* cq;    // kStages x 128 dh - query sums
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
  size_t oq = take(kStages * kTile, 1024), ok = take(kStages * kTile, 1024), ov = take(kStages * kTile, 1024);
  size_t op = take(2 * kTile, 1024);
  size_t oks = take(kStages * 128 * 4, 16), ocq = take(kStages * 128 * 4, 16);
  size_t orl = take(kMaxLen, 16);
  size_t ob = take((3 * kStages + 13) * 8, 8);
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
    s->empty = b + kStages;
    s->sums = b + 2 * kStages;
    uint64_t* d = b + 3 * kStages;  // double-buffered S / P / O barriers
    s->s_full = d + 0;
    s->s_empty = d + 2;
    s->p_full = d + 4;
    s->p_empty = d + 6;
    s->o_full = d + 8;
    s->o_empty = d + 10;
    s->drain = d + 12;
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
  }
  return off;
}

// bit 7 of each byte of the result is set when that byte of w is nonzero
// (adding 0x7F to the low seven bits carries into bit 7 exactly when they are
// not all zero; no carry crosses a byte)
__device__ __forceinline__ uint32_t byte_nonzero_msb(uint32_t w) {
  return (((w & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | w) & 0x80808080u;
}

// byte permute: result byte k is byte sel[4k+2:4k] of x, or that byte's sign bit
// replicated when sel bit 4k+3 is set
__device__ __forceinline__ uint32_t prmt_u32(uint32_t x, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %1, %2;" : "=r"(d) : "r"(x), "r"(sel));
  return d;
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

  // zero every operand buffer once: an unused slot of the last item then reads
  // finite data
  {
    uint4 z = make_uint4(0u, 0u, 0u, 0u);
    uint4* b = reinterpret_cast<uint4*>(sm.q);
    const int n = ((3 * kStages + 2) * kTile) / 16;  // q, k, v (kStages each) and p (2) are contiguous
    for (int i = threadIdx.x; i < n; i += kThreads) b[i] = z;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1 + kEpiWarps);
      mbar_init(&sm.sums[i], kEpiWarps);
    }
    for (int i = 0; i < 2; ++i) {
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
      int last_ph[kStages];
      for (int i = 0; i < kStages; ++i) last_ph[i] = -1;
      for (int g = 0; g < G; ++g) {
        const int s = g % kStages;
        const uint32_t ph = (uint32_t)(g / kStages) & 1u;
        if (!mbar_wait(&sm.empty[s], ph ^ 1u, 141)) { ok = false; break; }
        const int item = (int)blockIdx.x + (g / p.T) * (int)gridDim.x, t = g % p.T;
        const int nslots = (2 * item + 1 < BH) ? 2 : 1;
        mbar_expect_tx(&sm.full[s], (uint32_t)(3 * nslots * kHalf));
        last_ph[s] = (int)ph;
        for (int sl = 0; sl < nslots; ++sl) {
          const int bh = 2 * item + sl, b = bh / p.H, h = bh % p.H, z = t * p.B + b;
          // 4-D maps {dh, H, N, T*B}, box {64, 1, 64, 1}: d >= dh and rows >= N read as zero
          tma_load_4d(sm.q + s * kTile + sl * kHalf, &tmQ, &sm.full[s], 0, h, 0, z);
          tma_load_4d(sm.k + s * kTile + sl * kHalf, &tmK, &sm.full[s], 0, h, 0, z);
          tma_load_4d(sm.v + s * kTile + sl * kHalf, &tmV, &sm.full[s], 0, h, 0, z);
        }
      }
      if (!ok) {
        for (int i = 0; i < kStages; ++i)
          if (last_ph[i] >= 0) mbar_wait(&sm.full[i], (uint32_t)last_ph[i], 142);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    bool ok = true;
    const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
    const uint32_t idesc_pv = idesc_bf16_f32(128, 128, 0, 1);
    auto issue_s = [&](int g) -> bool {
      const int s = g & 1, qs = g % kStages;
      if (!mbar_wait(&sm.full[qs], (uint32_t)(g / kStages) & 1u, 151)) return false;
      if (!mbar_wait(&sm.s_empty[s], ((g >> 1) & 1) ^ 1u, 152)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sm.q + qs * kTile), ka = smem_u32(sm.k + qs * kTile);
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
      const int s = g & 1, qs = g % kStages;
      if (!mbar_wait(&sm.p_full[s], (g >> 1) & 1, 153)) { ok = false; break; }
      if (!mbar_wait(&sm.o_empty[s], ((g >> 1) & 1) ^ 1u, 154)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_u32(sm.p + s * kTile), va = smem_u32(sm.v + qs * kTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // keys 16 kk .. 16 kk + 15 of each slot; the two slots' V tiles are the
          // two 64-column atoms of B (kHalf bytes apart)
          const uint64_t adesc = umma_desc(pa + kk * 32, 16, 1024, 2);
          const uint64_t bdesc = umma_desc(va + kk * 2048, kHalf, 1024, 2);
          umma_bf16(tm_o + s * 128, adesc, bdesc, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.o_full[s]);
        umma_commit(&sm.p_empty[s]);
        umma_commit(&sm.empty[qs]);
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
    // the log-distance bias of this thread's row and 32 key columns: the same for
    // every unit, so it stays in registers, as fp32 pairs (XNOR form only)
    float2 rb2[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float r[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kj = kc0 + 2 * i + e;
        const int dist = qi > kj ? qi - kj : kj - qi;
        r[e] = (p.mode == 1 && dist < p.lmax) ? (float)sm.rl[dist] : 0.0f;
      }
      rb2[i] = make_float2(r[0], r[1]);
    }
    const bool mask_pf = p.mask_mode == 2 && p.mask_vec && kc0 + 32 <= p.Nk;
    // where a unit's rows go: step t, item (slot pair) and this thread's (batch,
    // head); advanced one unit at a time, with one division per item
    struct UnitPos {
      int t, item, b, h;
      bool valid;  // the slot exists and the row is a query
    };
    auto set_item = [&](UnitPos& u) {
      const int bh = 2 * u.item + slot;
      u.valid = bh < BH && qi < p.Nq;
      u.b = bh / p.H;
      u.h = bh - u.b * p.H;
    };
    auto advance = [&](UnitPos& u) {
      if (++u.t == p.T) {
        u.t = 0;
        u.item += (int)gridDim.x;
        set_item(u);
      }
    };
    UnitPos cur;
    cur.t = 0;
    cur.item = (int)blockIdx.x;
    set_item(cur);
    UnitPos nxt = cur, prv = cur;
    advance(nxt);
    // dense masks read as 16-byte vectors are loaded one unit ahead (the 32
    // mask bytes of this thread's row and key columns), so their latency
    // hides behind the previous unit's work
    auto mask_load = [&](const UnitPos& u, uint4& m0, uint4& m1) {
      m0 = make_uint4(0u, 0u, 0u, 0u);
      m1 = m0;
      if (u.valid) {
        const uint4* mrow = reinterpret_cast<const uint4*>(p.mask + u.t * p.m_st + u.b * p.m_sb + u.h * p.m_sh +
                                                           (int64_t)qi * p.m_sq + kc0);
        m0 = __ldg(mrow);
        m1 = __ldg(mrow + 1);
      }
    };
    // key sums (-|k_j|, first-half warps) and dh - |q_i| (second half) of unit gg
    // into its stage; the epilogue is then done with the stage's Q and K.  Run
    // one unit ahead, so that the all-warp barrier on the sums is met by the
    // time P needs them.
    auto sums = [&](int gg) -> bool {
      const int qs = gg % kStages;
      if (!mbar_wait(&sm.full[qs], (uint32_t)(gg / kStages) & 1u, 161)) return false;
      if (p.mode == 1) {
        if (half == 0)
          sm.ks[qs * 128 + row] = -(float)row_count_sw128(sm.k + qs * kTile, row, p.dh);
        else
          sm.cq[qs * 128 + row] = (float)(p.dh - row_count_sw128(sm.q + qs * kTile, row, p.dh));
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.empty[qs]);
        if (p.mode == 1) mbar_arrive(&sm.sums[qs]);
      }
      return true;
    };
    uint4 pm0 = make_uint4(0u, 0u, 0u, 0u), pm1 = pm0;
    if (mask_pf && G > 0) mask_load(cur, pm0, pm1);
    const float2 two2 = make_float2(2.0f, 2.0f), scale2 = make_float2(scale, scale);
    const float2 gain2 = make_float2(p.gain, p.gain), beta2 = make_float2(beta, beta);
    bool ok = G == 0 || sums(0);
    for (int g = 0; g <= G && ok; ++g) {
      if (g < G) {
        // ---- build P of unit g
        const int s = g & 1, qs = g % kStages;
        const uint32_t qph = (uint32_t)(g / kStages) & 1u;
        // keep flags of this thread's 32 key columns: the most significant bit of
        // byte i of fw[i / 4] is set when key kc0 + i is kept
        uint32_t fw[8];
        if (mask_pf) {
          const uint32_t w[8] = {pm0.x, pm0.y, pm0.z, pm0.w, pm1.x, pm1.y, pm1.z, pm1.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) fw[k] = byte_nonzero_msb(w[k]);
          if (g + 1 < G) mask_load(nxt, pm0, pm1);
        } else {
          uint32_t mbits = 0xffffffffu;  // keep bit per key column of this warp
          if (p.mask_mode == 2) {
            mbits = 0u;
            if (cur.valid) {
              const uint8_t* mrow =
                  p.mask + cur.t * p.m_st + cur.b * p.m_sb + cur.h * p.m_sh + (int64_t)qi * p.m_sq + kc0;
              for (int i = 0; i < 32 && kc0 + i < p.Nk; ++i) mbits |= (mrow[i] != 0 ? 1u : 0u) << i;
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
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // bit j of the nibble to bit 7 of byte j (the shifted copies do not overlap)
            const uint32_t x = (mbits >> (4 * k)) & 0xFu;
            fw[k] = ((x * 0x00204081u) & 0x01010101u) << 7;
          }
        }
        if (p.mode == 1 && !mbar_wait(&sm.sums[qs], qph, 162)) { ok = false; break; }
        if (!mbar_wait(&sm.s_full[s], (g >> 1) & 1, 163)) { ok = false; break; }
        if (!mbar_wait(&sm.p_empty[s], ((g >> 1) & 1) ^ 1u, 164)) { ok = false; break; }
        tc_fence_after();
        uint32_t raw[32];
        tmem_ld32_raw(tm_s + s * 128 + lane_off + slot * 64 + kc0, raw);
        const float c_row = p.mode == 1 ? sm.cq[qs * 128 + row] : 0.0f;
        const float2 c2 = make_float2(c_row, c_row);
        const float* nks = sm.ks + qs * 128 + slot * 64 + kc0;  // -|k_j|
        tmem_wait_ld_fence32(raw);
        // S' = 2 S + (c_i + R_ij - |k_j|) in packed fp32 pairs (all integers, exact), then
        // bf16 pairs (exact: |S'| < 256) with the masked keys cleared
        uint32_t pw[16];
#pragma unroll
        for (int i0 = 0; i0 < 16; i0 += 2) {
          // four key sums in one 16-byte load (the same address in every lane)
          const float4 k4 = p.mode == 1 ? *reinterpret_cast<const float4*>(nks + 2 * i0)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int i = i0 + u;
            float2 sc = make_float2(__uint_as_float(raw[2 * i]), __uint_as_float(raw[2 * i + 1]));
            if (p.mode == 1) {
              const float2 nk2 = u == 0 ? make_float2(k4.x, k4.y) : make_float2(k4.z, k4.w);
              sc = fma2(sc, two2, add2(add2(rb2[i], c2), nk2));
            }
            // keep masks of keys 2i, 2i+1 as 0xFFFF halves (sign replication of the flags)
            const uint32_t keep = prmt_u32(fw[i >> 1], (i & 1) ? 0xBBAAu : 0x9988u);
            pw[i] = pack_bf16x2(sc.x, sc.y) & keep;
          }
        }
        // 32 keys of row `row` into the 64-key atom (K-major, 128-byte swizzle)
        uint8_t* prow = sm.p + s * kTile + row * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int ch = half * 4 + c;
          *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) =
              make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.s_empty[s]);
          mbar_arrive(&sm.p_full[s]);
        }
        if (g + 1 < G && !sums(g + 1)) { ok = false; break; }
      }
      if (g >= 1) {
        // ---- spikes of unit g - 1
        const int u = g - 1, s = u & 1;
        if (!mbar_wait(&sm.o_full[s], (u >> 1) & 1, 165)) { ok = false; break; }
        tc_fence_after();
        uint32_t raw[32];
        tmem_ld32_raw(tm_o + s * 128 + lane_off + slot * 64 + dcol0, raw);
        tmem_wait_ld_fence32(raw);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_empty[s]);
        if (prv.t == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mem[i] = 0.0f;
        }
        if (prv.valid) {
          const int64_t obase = (((int64_t)prv.t * p.B + prv.b) * p.Nq + qi) * D + (int64_t)prv.h * p.dh + dcol0;
          float* aout = p.attn_out ? p.attn_out + ((((int64_t)prv.t * p.B + prv.b) * p.H + prv.h) * p.Nq + qi) * p.dh +
                                         dcol0
                                   : nullptr;
#pragma unroll
          for (int d0 = 0; d0 < 32; d0 += 8) {
            if (d0 < dcols) {
              // a = scale O, LIF over t: packed fp32 pairs that round as the scalar
              // reference (a * gain is exact when the gain is 1)
              uint32_t bits[4];
#pragma unroll
              for (int j = 0; j < 8; j += 2) {
                const int dd = d0 + j;
                const float2 a = mul2(make_float2(__uint_as_float(raw[dd]), __uint_as_float(raw[dd + 1])), scale2);
                if (aout) *reinterpret_cast<float2*>(aout + dd) = a;
                const float2 uu = add2(mul2(make_float2(mem[dd], mem[dd + 1]), beta2), mul2(a, gain2));
                const bool f0 = uu.x > vth, f1 = uu.y > vth;
                mem[dd] = f0 ? vr : uu.x;
                mem[dd + 1] = f1 ? vr : uu.y;
                bits[j >> 1] = (f0 ? 0x3F80u : 0u) | (f1 ? 0x3F800000u : 0u);
              }
              if (p.out_bf16)
                *reinterpret_cast<uint4*>(p.out_bf16 + obase + d0) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
              if (p.out_f32) {
                float4 lo, hi;
                lo.x = (bits[0] & 0xFFFFu) ? 1.0f : 0.0f; lo.y = (bits[0] >> 16) ? 1.0f : 0.0f;
                lo.z = (bits[1] & 0xFFFFu) ? 1.0f : 0.0f; lo.w = (bits[1] >> 16) ? 1.0f : 0.0f;
                hi.x = (bits[2] & 0xFFFFu) ? 1.0f : 0.0f; hi.y = (bits[2] >> 16) ? 1.0f : 0.0f;
                hi.z = (bits[3] & 0xFFFFu) ? 1.0f : 0.0f; hi.w = (bits[3] >> 16) ? 1.0f : 0.0f;
                *reinterpret_cast<float4*>(p.out_f32 + obase + d0) = lo;
                *reinterpret_cast<float4*>(p.out_f32 + obase + d0 + 4) = hi;
              }
            }
          }
        }
      }
      prv = cur;
      cur = nxt;
      advance(nxt);
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
