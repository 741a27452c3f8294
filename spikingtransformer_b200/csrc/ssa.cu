// Spiking self-attention on spike tensors, without softmax, on tcgen05.
//
// Reference (flofiz/SpikingTransformer):
//   XNOR variant   SSA.py:145-165 (Dh - Hamming distance), :177-201 (log-
//                  distance bias), :234-244 (+bias, *mask, (*scale) @ V, LIF)
//   plain variant  SSA.py:81-86 ((Q K^T) * mask) @ V * 0.125, LIF)
//
// Q, K, V are {0,1} spikes in bf16, [T][B][N][H*dh] (head-merged, t-major).
// One CTA owns (b, h, a block of 128 queries) and walks t = 0..T-1:
//   S   = Q K^T            tcgen05.mma kind::f16, fp32 accumulate in TMEM
//                          (integer counts <= dh: exact)
//   P   = transform(S)     epilogue warps: XNOR score dh - (|q|+|k|-2S) + R,
//                          mask, written as bf16 integers (<= 255: exact) into
//                          a 128-byte-swizzled K-major tile in shared memory
//   O  += P V              tcgen05.mma with V as an MN-major operand
//                          (integer sums < 2^24: exact)
//   a   = scale * O        fp32; then LIF (v_th of lifs) over t in registers
// Keys are processed in blocks of 128 with S double-buffered in TMEM, so
// the transform of one block overlaps the Q K^T of the next.
//
// The spike-count product O is exact.  The reference rounds S*scale per
// element before the @V (SSA.py:242); here the scale is applied once to the
// exact integer sum, a difference of a few ulp in the LIF input.
#include <cstdlib>

#include "common.cuh"

namespace spk {
namespace ssak {

constexpr int kThreads = 192;
constexpr int kEpi = 128;
constexpr int kKB = 128;          // keys per block
constexpr int kTile = 128 * 128;  // 128 rows x 128 bytes
constexpr int kMaxLen = 8192;     // longest sequence (log-distance table size)

struct Params {
  int T, B, H, Nq, Nk, dh;
  int mode;       // 0 plain, 1 xnor
  int mask_mode;  // 0 none, 1 causal (key <= query), 2 dense u8
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
  int q_blocks;
  int lmax;                 // max(Nq, Nk)
};

struct Smem {
  uint8_t* q;   // 2 x kTile
  uint8_t* k;   // 2 x kTile
  uint8_t* v;   // 2 x kTile
  uint8_t* p;   // 2 x (2 x kTile)  (128 rows x 128 keys bf16 = two 64-key atoms)
  float* ks;    // 2 x 128
  uint8_t* rl;  // log-distance table [lmax]
  uint64_t *q_full, *q_empty, *kv_full, *kv_empty, *s_full, *s_empty, *p_full, *p_empty;
  uint64_t *o_full, *o_empty, *drain;
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
  size_t oq = take(2 * kTile, 1024), ok = take(2 * kTile, 1024), ov = take(2 * kTile, 1024);
  size_t op = take(4 * kTile, 1024);
  size_t oks = take(2 * 128 * 4, 16);
  size_t orl = take((size_t)lmax, 16);
  size_t ob = take(20 * 8, 8);
  size_t otm = take(4, 4);
  if (s) {
    s->q = base + oq;
    s->k = base + ok;
    s->v = base + ov;
    s->p = base + op;
    s->ks = reinterpret_cast<float*>(base + oks);
    s->rl = base + orl;
    uint64_t* b = reinterpret_cast<uint64_t*>(base + ob);
    s->q_full = b + 0;
    s->q_empty = b + 2;
    s->kv_full = b + 4;
    s->kv_empty = b + 6;
    s->s_full = b + 8;
    s->s_empty = b + 10;
    s->p_full = b + 12;
    s->p_empty = b + 14;
    s->o_full = b + 16;
    s->o_empty = b + 17;
    s->drain = b + 18;
    s->tmem_base = reinterpret_cast<uint32_t*>(base + otm);
  }
  return off + 1024;
}

// number of key blocks processed for query block starting at q0
__device__ __forceinline__ int key_blocks(const Params& p, int q0) {
  int nk = p.Nk;
  if (p.mask_mode == 1) {
    const int last_q = min(q0 + 127, p.Nq - 1);
    nk = min(nk, last_q + 1);  // keys beyond the last query are all masked
  }
  return (nk + kKB - 1) / kKB;
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

__global__ void __launch_bounds__(kThreads, 1)
    ssa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const Params p) {
  // dynamic shared memory, 1024-byte aligned (128-byte swizzle atoms); pointers derived from
  // it by plain arithmetic so the compiler keeps them in the shared address space
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  Smem sm;
  smem_layout(p.lmax, base, &sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qblk = blockIdx.x % p.q_blocks;
  const int bh = blockIdx.x / p.q_blocks;
  const int h = bh % p.H, b = bh / p.H;
  const int q0 = qblk * 128;
  const int nkb = key_blocks(p, q0);
  const int dsteps = (p.dh + 15) >> 4;       // K steps of Q K^T
  const int dpad = dsteps * 16;              // N of P V

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1 + 4);
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1 + 4);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], 4);
      mbar_init(&sm.p_full[i], 4);
      mbar_init(&sm.p_empty[i], 1);
    }
    mbar_init(sm.o_full, 1);
    mbar_init(sm.o_empty, 4);
    mbar_init(sm.drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_base, 512);
    tmem_relinquish();
  }
  // log-distance bias table R[d] = smallest k >= 0 with (d+1) * 2^k >= L-1
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  const uint32_t tm_s0 = tmem, tm_o = tmem + 256;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int kv_it = 0;
      bool ok = true;
      int q_ph[2] = {-1, -1}, kv_ph[2] = {-1, -1};  // phase of the last load issued per buffer
      for (int t = 0; t < p.T && ok; ++t) {
        const int qb = t & 1;
        if (!mbar_wait(&sm.q_empty[qb], ((t >> 1) & 1) ^ 1u, 41)) { ok = false; break; }
        mbar_expect_tx(&sm.q_full[qb], kTile);
        q_ph[qb] = (t >> 1) & 1;
        // 4-D maps {dh, H, N, T*B}: the box {64, 1, 128, 1} zero-fills d >= dh
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(sm.q + qb * kTile)),
            "l"(&tmQ), "r"(smem_u32(&sm.q_full[qb])), "r"(0), "r"(h), "r"(q0), "r"(t * p.B + b)
            : "memory");
        for (int kb = 0; kb < nkb; ++kb, ++kv_it) {
          const int s = kv_it & 1;
          if (!mbar_wait(&sm.kv_empty[s], ((kv_it >> 1) & 1) ^ 1u, 42)) { ok = false; break; }
          mbar_expect_tx(&sm.kv_full[s], 2 * kTile);
          kv_ph[s] = (kv_it >> 1) & 1;
          asm volatile(
              "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(sm.k + s * kTile)),
              "l"(&tmK), "r"(smem_u32(&sm.kv_full[s])), "r"(0), "r"(h), "r"(kb * kKB), "r"(t * p.B + b)
              : "memory");
          asm volatile(
              "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(sm.v + s * kTile)),
              "l"(&tmV), "r"(smem_u32(&sm.kv_full[s])), "r"(0), "r"(h), "r"(kb * kKB), "r"(t * p.B + b)
              : "memory");
        }
      }
      if (!ok) {
        // wait (bounded) for loads that may still be landing in shared memory
        for (int i = 0; i < 2; ++i) {
          if (q_ph[i] >= 0) mbar_wait(&sm.q_full[i], (uint32_t)q_ph[i], 43);
          if (kv_ph[i] >= 0) mbar_wait(&sm.kv_full[i], (uint32_t)kv_ph[i], 43);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    int kv_qk = 0, kv_pv = 0, s_it = 0, p_it = 0;
    bool ok = true;
    const uint32_t idesc_pv = idesc_bf16_f32(128, dpad, 0, 1);
    auto issue_qk = [&](int kb, int qb) -> bool {
      const int s = kv_qk & 1, sb = s_it & 1;
      if (!mbar_wait(&sm.kv_full[s], (kv_qk >> 1) & 1, 51)) return false;
      if (!mbar_wait(&sm.s_empty[sb], ((s_it >> 1) & 1) ^ 1u, 52)) return false;
      tc_fence_after();
      if (lane == 0) {
        const int ncols = min(kKB, ((p.Nk - kb * kKB) + 15) / 16 * 16);
        const uint32_t idesc = idesc_bf16_f32(128, ncols, 0, 0);
        const uint32_t qa = smem_u32(sm.q + qb * kTile), ka = smem_u32(sm.k + s * kTile);
        for (int kk = 0; kk < dsteps; ++kk)
          umma_bf16(tm_s0 + sb * kKB, umma_desc(qa + kk * 32, 16, 1024, 2), umma_desc(ka + kk * 32, 16, 1024, 2),
                    idesc, kk > 0 ? 1u : 0u);
        umma_commit(&sm.s_full[sb]);
      }
      __syncwarp();
      ++kv_qk;
      ++s_it;
      return true;
    };
    for (int t = 0; t < p.T && ok; ++t) {
      const int qb = t & 1;
      if (!mbar_wait(&sm.q_full[qb], (t >> 1) & 1, 53)) { ok = false; break; }
      tc_fence_after();
      if (nkb > 0 && !issue_qk(0, qb)) { ok = false; break; }
      for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb && !issue_qk(kb + 1, qb)) { ok = false; break; }
        const int pb = p_it & 1, s = kv_pv & 1;
        if (!mbar_wait(&sm.p_full[pb], (p_it >> 1) & 1, 54)) { ok = false; break; }
        if (kb == 0 && !mbar_wait(sm.o_empty, (t & 1) ^ 1u, 55)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const int ncols = min(kKB, ((p.Nk - kb * kKB) + 15) / 16 * 16);
          const uint32_t pa = smem_u32(sm.p + pb * 2 * kTile), va = smem_u32(sm.v + s * kTile);
          for (int kk = 0; kk < ncols / 16; ++kk) {
            const uint64_t adesc = umma_desc(pa + (kk >> 2) * kTile + (kk & 3) * 32, 16, 1024, 2);
            const uint64_t bdesc = umma_desc(va + kk * 2048, kTile, 1024, 2);
            umma_bf16(tm_o, adesc, bdesc, idesc_pv, (kb | kk) ? 1u : 0u);
          }
          umma_commit(&sm.p_empty[pb]);
          umma_commit(&sm.kv_empty[s]);
        }
        __syncwarp();
        ++p_it;
        ++kv_pv;
      }
      if (!ok) break;
      if (lane == 0) {
        umma_commit(sm.o_full);
        umma_commit(&sm.q_empty[qb]);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) umma_commit(sm.drain);
      __syncwarp();
      mbar_wait(sm.drain, 0, 56);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // query row within the block
    const int qi = q0 + row;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float scale = __ldg(p.scale);
    const float beta = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
    const int D = p.H * p.dh;
    float mem[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) mem[i] = 0.0f;
    int kv_it = 0, s_it = 0, p_it = 0;
    bool ok = true;
    for (int t = 0; t < p.T && ok; ++t) {
      const int qb = t & 1;
      if (!mbar_wait(&sm.q_full[qb], (t >> 1) & 1, 61)) { ok = false; break; }
      float c_row = 0.0f;  // dh - |q_i|
      if (p.mode == 1) c_row = (float)p.dh - row_sum_sw128(sm.q + qb * kTile, row, p.dh);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_empty[qb]);
      for (int kb = 0; kb < nkb; ++kb, ++kv_it, ++s_it, ++p_it) {
        const int s = kv_it & 1, sb = s_it & 1, pb = p_it & 1;
        if (!mbar_wait(&sm.kv_full[s], (kv_it >> 1) & 1, 62)) { ok = false; break; }
        float* ks = sm.ks + s * 128;
        if (p.mode == 1) ks[row] = row_sum_sw128(sm.k + s * kTile, row, p.dh);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.kv_empty[s]);
        named_bar_sync(1, kEpi);  // all key sums of this block are in place
        if (!mbar_wait(&sm.s_full[sb], (s_it >> 1) & 1, 63)) { ok = false; break; }
        if (!mbar_wait(&sm.p_empty[pb], ((p_it >> 1) & 1) ^ 1u, 64)) { ok = false; break; }
        tc_fence_after();
        const int k0 = kb * kKB;
        const int ncols = min(kKB, ((p.Nk - k0) + 15) / 16 * 16);
        uint8_t* ptile = sm.p + pb * 2 * kTile;
        const uint8_t* mrow = nullptr;
        if (p.mask_mode == 2 && qi < p.Nq)
          mrow = p.mask + t * p.m_st + b * p.m_sb + h * p.m_sh + (int64_t)qi * p.m_sq;
        for (int c0 = 0; c0 < ncols; c0 += 32) {
          float v[32];
          if (c0 + 32 <= ncols) {
            tmem_ld32(tm_s0 + sb * kKB + lane_off + c0, v);
          } else {
            tmem_ld16(tm_s0 + sb * kKB + lane_off + c0, v);
#pragma unroll
            for (int i = 16; i < 32; ++i) v[i] = 0.0f;
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kj = k0 + c0 + i;
            float sc = v[i];
            if (p.mode == 1) {
              const int dist = qi > kj ? qi - kj : kj - qi;
              const float rb = (dist < p.lmax) ? (float)sm.rl[dist] : 0.0f;
              sc = fmaf(2.0f, sc, c_row - ks[c0 + i]) + rb;
            }
            bool keep = kj < p.Nk;
            if (p.mask_mode == 1) keep = keep && (kj <= qi);
            else if (p.mask_mode == 2) keep = keep && mrow != nullptr && __ldg(mrow + kj) != 0;
            v[i] = keep ? sc : 0.0f;
          }
          // write 32 keys of row `row` into the K-major swizzled P tile
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int j = c0 + g * 8;
            {
              const int atom = j >> 6, ch = (j & 63) >> 3;
              uint4 w;
              w.x = pack_bf16x2(v[g * 8 + 0], v[g * 8 + 1]);
              w.y = pack_bf16x2(v[g * 8 + 2], v[g * 8 + 3]);
              w.z = pack_bf16x2(v[g * 8 + 4], v[g * 8 + 5]);
              w.w = pack_bf16x2(v[g * 8 + 6], v[g * 8 + 7]);
              *reinterpret_cast<uint4*>(ptile + atom * kTile + row * 128 + ((ch ^ (row & 7)) << 4)) = w;
            }
          }
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.s_empty[sb]);
          mbar_arrive(&sm.p_full[pb]);
        }
      }
      if (!ok) break;
      // ---- output of step t: scale, LIF, spikes
      if (!mbar_wait(sm.o_full, t & 1, 65)) { ok = false; break; }
      tc_fence_after();
      float o[64];
      for (int c0 = 0; c0 < dpad; c0 += 16) tmem_ld16(tm_o + lane_off + c0, o + c0);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sm.o_empty);
      if (qi < p.Nq) {
        const int64_t obase = (((int64_t)t * p.B + b) * p.Nq + qi) * D + (int64_t)h * p.dh;
        float* aout = p.attn_out ? p.attn_out + ((((int64_t)t * p.B + b) * p.H + h) * p.Nq + qi) * p.dh : nullptr;
#pragma unroll
        for (int d0 = 0; d0 < 64; d0 += 8) {
          if (d0 < p.dh) {
            float sp[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float a = __fmul_rn(o[d0 + i], scale);
              if (aout) aout[d0 + i] = a;
              const float cur = p.gain != 1.0f ? __fmul_rn(a, p.gain) : a;
              const float u = __fadd_rn(__fmul_rn(mem[d0 + i], beta), cur);
              const bool fire = u > vth;
              sp[i] = fire ? 1.0f : 0.0f;
              mem[d0 + i] = fire ? vr : u;
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
    (void)ok;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace ssak

SPK_DEFINE_ERROR_READER(ssa_read_device_error)

using namespace ssak;

// score-free kernel for unmasked attention (ssa_lin.cu)
int launch_ssa_lin(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, int T, int B, int H,
                   int Nq, int Nk, int dh, int variant, const float* scale, const float* lif_beta,
                   const float* lif_vth, const float* lif_vr, float gain, void* out_bf16, float* out_f32,
                   float* attn_out, bool attn_token_major, cudaStream_t st);

// two (batch, head) pairs per tile for Nq, Nk <= 64 (ssa_short.cu)
int launch_ssa_short(const void* q, const void* k, const void* v, int T, int B, int H, int Nq, int Nk, int dh,
                     int variant, int mask_mode, const uint8_t* mask, int64_t m_st, int64_t m_sb, int64_t m_sh,
                     int64_t m_sq, const float* scale, const float* lif_beta, const float* lif_vth,
                     const float* lif_vr, float gain, void* out_bf16, float* out_f32, float* attn_out,
                     cudaStream_t st);

static bool force_dense() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SPK_SSA_DENSE");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

static int make_qkv_map(CUtensorMap* m, const void* ptr, int dh, int H, int N, int TB) {
  uint64_t dims[4] = {(uint64_t)dh, (uint64_t)H, (uint64_t)N, (uint64_t)TB};
  uint64_t strides[3] = {(uint64_t)dh * 2, (uint64_t)H * dh * 2, (uint64_t)N * H * dh * 2};
  uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(m, ptr, 4, dims, strides, box, true);
}

// q / k / v as [T*B][H][N][dh] views with element strides (t*b, head,
// position) and unit stride along dh
static int make_heads_map(CUtensorMap* m, const void* ptr, int dh, int H, int N, int TB, const int64_t* st) {
  uint64_t dims[4] = {(uint64_t)dh, (uint64_t)H, (uint64_t)N, (uint64_t)TB};
  uint64_t strides[3] = {(uint64_t)st[1] * 2, (uint64_t)st[2] * 2, (uint64_t)st[0] * 2};
  uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(m, ptr, 4, dims, strides, box, true);
}

}  // namespace spk

extern "C" {

int spk_ssa_fwd_heads(const void* q, const void* k, const void* v, const int64_t* strides, int variant,
                      const float* scale, const float* lif_beta, const float* lif_vth, const float* lif_vreset,
                      float in_gain, int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, void* out,
                      int out_dtype, float* attn_out, void* stream) {
  using namespace spk;
  SPK_REQUIRE(q && k && v && strides && out && scale && lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID,
              "null pointer argument");
  SPK_REQUIRE(variant == 0 || variant == 1, SPK_ERR_INVALID, "variant must be 0 (plain) or 1 (xnor)");
  SPK_REQUIRE(out_dtype == SPK_BF16 || out_dtype == SPK_F32, SPK_ERR_INVALID, "out dtype must be bf16 or f32");
  SPK_REQUIRE(dh >= 8 && dh <= 64 && dh % 8 == 0, SPK_ERR_SHAPE, "head dim %lld unsupported (8..64, multiple of 8)",
              (long long)dh);
  SPK_REQUIRE(T >= 1 && B >= 1 && H >= 1 && Nq >= 1 && Nk >= 1 && Nq <= 256 && Nk <= 256, SPK_ERR_SHAPE,
              "unsupported sizes T=%lld B=%lld H=%lld Nq=%lld Nk=%lld (Nq, Nk <= 256)", (long long)T, (long long)B,
              (long long)H, (long long)Nq, (long long)Nk);
  SPK_REQUIRE(T * B < (1ll << 31) && B * H < (1ll << 31), SPK_ERR_SHAPE, "grid too large");
  for (int i = 0; i < 9; ++i)
    SPK_REQUIRE(strides[i] > 0 && (strides[i] * 2) % 16 == 0, SPK_ERR_ALIGN,
                "operand strides must be positive multiples of 8 elements (stride %d = %lld)", i,
                (long long)strides[i]);
  SPK_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16), SPK_ERR_ALIGN,
              "q, k, v and out must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  CUtensorMap tq, tk, tv;
  const int TB = (int)(T * B);
  if ((rc = make_heads_map(&tq, q, (int)dh, (int)H, (int)Nq, TB, strides)) != SPK_OK) return rc;
  if ((rc = make_heads_map(&tk, k, (int)dh, (int)H, (int)Nk, TB, strides + 3)) != SPK_OK) return rc;
  if ((rc = make_heads_map(&tv, v, (int)dh, (int)H, (int)Nk, TB, strides + 6)) != SPK_OK) return rc;
  rc = launch_ssa_lin(tq, tk, tv, (int)T, (int)B, (int)H, (int)Nq, (int)Nk, (int)dh, variant, scale, lif_beta,
                      lif_vth, lif_vreset, in_gain, out_dtype == SPK_BF16 ? out : nullptr,
                      out_dtype == SPK_F32 ? reinterpret_cast<float*>(out) : nullptr, attn_out, true,
                      reinterpret_cast<cudaStream_t>(stream));
  if (rc != SPK_OK) return rc;
  return check_launch("ssa_lin_kernel");
}

int spk_ssa_fwd(const void* q, const void* k, const void* v, int variant, int mask_mode, const uint8_t* mask,
                int64_t mask_stride_t, int64_t mask_stride_b, int64_t mask_stride_h, int64_t mask_stride_q,
                const float* scale, const float* lif_beta, const float* lif_vth, const float* lif_vreset,
                float in_gain, int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, void* out,
                int out_dtype, float* attn_out, void* stream) {
  using namespace spk;
  SPK_REQUIRE(q && k && v && out && scale && lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID,
              "null pointer argument");
  SPK_REQUIRE(variant == 0 || variant == 1, SPK_ERR_INVALID, "variant must be 0 (plain) or 1 (xnor)");
  SPK_REQUIRE(mask_mode >= 0 && mask_mode <= 2 && (mask_mode != 2 || mask), SPK_ERR_INVALID, "bad mask");
  SPK_REQUIRE(out_dtype == SPK_BF16 || out_dtype == SPK_F32, SPK_ERR_INVALID, "out dtype must be bf16 or f32");
  SPK_REQUIRE(dh >= 8 && dh <= 64 && dh % 8 == 0, SPK_ERR_SHAPE, "head dim %lld unsupported (8..64, multiple of 8)",
              (long long)dh);
  SPK_REQUIRE(T >= 1 && B >= 1 && H >= 1 && Nq >= 1 && Nk >= 1 && Nq <= kMaxLen && Nk <= kMaxLen, SPK_ERR_SHAPE,
              "unsupported sizes T=%lld B=%lld H=%lld Nq=%lld Nk=%lld", (long long)T, (long long)B, (long long)H,
              (long long)Nq, (long long)Nk);
  SPK_REQUIRE(T * B < (1ll << 31) && (Nq + 127) / 128 * B * H < (1ll << 31), SPK_ERR_SHAPE, "grid too large");
  SPK_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16), SPK_ERR_ALIGN,
              "q, k, v and out must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_qkv_map(&tq, q, (int)dh, (int)H, (int)Nq, (int)(T * B))) != SPK_OK) return rc;
  if ((rc = make_qkv_map(&tk, k, (int)dh, (int)H, (int)Nk, (int)(T * B))) != SPK_OK) return rc;
  if ((rc = make_qkv_map(&tv, v, (int)dh, (int)H, (int)Nk, (int)(T * B))) != SPK_OK) return rc;
  if (mask_mode == 0 && !force_dense()) {
    rc = launch_ssa_lin(tq, tk, tv, (int)T, (int)B, (int)H, (int)Nq, (int)Nk, (int)dh, variant, scale, lif_beta,
                        lif_vth, lif_vreset, in_gain, out_dtype == SPK_BF16 ? out : nullptr,
                        out_dtype == SPK_F32 ? reinterpret_cast<float*>(out) : nullptr, attn_out, false,
                        reinterpret_cast<cudaStream_t>(stream));
    if (rc == SPK_OK) return check_launch("ssa_lin_kernel");
    if (rc != SPK_ERR_UNSUPPORTED) return rc;
  }
  if (Nq <= 64 && Nk <= 64 && !force_dense()) {
    rc = launch_ssa_short(q, k, v, (int)T, (int)B, (int)H, (int)Nq, (int)Nk, (int)dh, variant, mask_mode, mask,
                          mask_stride_t, mask_stride_b, mask_stride_h, mask_stride_q, scale, lif_beta, lif_vth,
                          lif_vreset, in_gain, out_dtype == SPK_BF16 ? out : nullptr,
                          out_dtype == SPK_F32 ? reinterpret_cast<float*>(out) : nullptr, attn_out,
                          reinterpret_cast<cudaStream_t>(stream));
    if (rc != SPK_ERR_UNSUPPORTED) return rc;
  }
  Params p = {};
  p.T = (int)T;
  p.B = (int)B;
  p.H = (int)H;
  p.Nq = (int)Nq;
  p.Nk = (int)Nk;
  p.dh = (int)dh;
  p.mode = variant;
  p.mask_mode = mask_mode;
  p.mask = mask;
  p.m_st = mask_stride_t;
  p.m_sb = mask_stride_b;
  p.m_sh = mask_stride_h;
  p.m_sq = mask_stride_q;
  p.scale = scale;
  p.lif_beta = lif_beta;
  p.lif_vth = lif_vth;
  p.lif_vr = lif_vreset;
  p.gain = in_gain;
  p.out_bf16 = out_dtype == SPK_BF16 ? reinterpret_cast<__nv_bfloat16*>(out) : nullptr;
  p.out_f32 = out_dtype == SPK_F32 ? reinterpret_cast<float*>(out) : nullptr;
  p.attn_out = attn_out;
  p.q_blocks = (int)((Nq + 127) / 128);
  p.lmax = (int)(Nq > Nk ? Nq : Nk);
  size_t smem = smem_layout(p.lmax, nullptr, nullptr);
  cudaError_t e = cudaFuncSetAttribute(ssa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int grid = (int)(B * H * p.q_blocks);
  ssa_kernel<<<grid, kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return check_launch("ssa_kernel");
}

}  // extern "C"
