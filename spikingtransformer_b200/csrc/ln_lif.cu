// LayerNorm -> LIF for training: forward and backward fused over the T steps
// of each token, with the Linear left to the library GEMM.
//
// Reference composition (flofiz/SpikingTransformer): nn.LayerNorm followed by
// the LIF module (SSA.py:218-228, :247-249; SpikingMLP.py:31-36), whose
// backward is LIFLayer.backward (Lif.py:46-102) and torch's LayerNorm
// backward.  Layout: pre-activations, spikes and gradients are
// [T][R][D] (t-major fold, R tokens, D features); LayerNorm runs over D for
// each of the T*R rows; the LIF couples the T rows of a token.
//
// Forward, per token: the T rows are loaded once into registers (D/(32 NW)
// columns per thread, NW warps per token), mean and variance by two passes
// (warp shuffles, plus shared memory when NW > 1), y = (x - mean) rstd gamma
// + beta, then the LIF over t with v = beta v + gain y (separately rounded
// multiply and add, as the reference), s = v > v_th, v = s ? v_reset : v.
// Spikes are written and (mean, rstd) of every row is saved.
//
// Backward, per token: x^ and the membrane are recomputed from the saved
// statistics; BPTT over t with the surrogate (SuperSpike or arctan) gives
// dL/dy; then the LayerNorm input gradient
//   dx = rstd (g - mean(g) - x^ mean(g x^)),  g = gamma dL/dy
// and per-column partial sums of dL/dgamma = sum dL/dy x^ and
// dL/dbeta = sum dL/dy, plus the LIF beta gradient sum g_v v_prev, are kept
// per block and reduced in a fixed order by a second kernel.
#include "common.cuh"

namespace spk {
namespace lnlif {

constexpr int kThreads = 128;  // 4 warps
constexpr int kMaxCpt = 16;    // columns per thread
constexpr int kMaxT = 4;

struct FwdParams {
  const void* pre;
  int pre_dtype;
  const float* gamma;
  const float* beta_ln;
  float eps;
  const float *lif_beta, *lif_vth, *lif_vr;
  float gain;
  void* spikes;
  int spike_dtype;
  float2* stats;  // [T*R] (mean, rstd)
  int T;
  int64_t R;
  int D, cpt;
};

struct BwdParams {
  const void* g_spikes;
  int gs_dtype;
  const void* pre;
  int pre_dtype;
  const float2* stats;
  const float* gamma;
  const float* beta_ln;
  const float *lif_beta, *lif_vth, *lif_vr;
  float gain;
  int surrogate;
  float k, c_arctan;
  void* g_pre;  // same dtype as pre
  float* part;  // [grid][2 D + 1]: dgamma partials, dbeta partials, LIF beta partial
  int T;
  int64_t R;
  int D, cpt;
};

__device__ __forceinline__ float load_elem(const void* p, int dt, int64_t i) {
  if (dt == SPK_F32) return reinterpret_cast<const float*>(p)[i];
  if (dt == SPK_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_elem(void* p, int dt, int64_t i, float v) {
  if (dt == SPK_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dt == SPK_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dt == SPK_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<uint8_t*>(p)[i] = v != 0.0f ? 1 : 0;
}

// four consecutive elements starting at i (16-byte aligned for fp32, 8 for 16-bit types)
__device__ __forceinline__ void load4(const void* p, int dt, int64_t i, float* o) {
  if (dt == SPK_F32) {
    const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  } else {
    const uint2 w = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
    if (dt == SPK_F16) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
      o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
    } else {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
    }
  }
}

__device__ __forceinline__ void store4(void* p, int dt, int64_t i, const float* v) {
  if (dt == SPK_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else if (dt == SPK_F16) {
    __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) = w;
  } else if (dt == SPK_BF16) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) = w;
  } else {
    uchar4 w = make_uchar4(v[0] != 0.0f, v[1] != 0.0f, v[2] != 0.0f, v[3] != 0.0f);
    *reinterpret_cast<uchar4*>(reinterpret_cast<uint8_t*>(p) + i) = w;
  }
}

// column of this thread's i-th element: V = 1 -> lanes interleave single columns;
// V = 4 -> each thread owns groups of four consecutive columns (vector loads)
template <int NW, int V>
__device__ __forceinline__ int col_of(int i, int wt, int lane) {
  if constexpr (V == 1) return wt * 32 + lane + i * 32 * NW;
  return ((i >> 2) * 32 * NW + wt * 32 + lane) * 4 + (i & 3);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// sums of vals[0..T) over the NW warps of one token (every thread gets the totals)
template <int NW>
__device__ __forceinline__ void token_sums(float (&vals)[kMaxT], int T, float* red, int wt) {
#pragma unroll
  for (int t = 0; t < kMaxT; ++t)
    if (t < T) vals[t] = warp_sum(vals[t]);
  if constexpr (NW > 1) {
    const int lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < kMaxT; ++t)
        if (t < T) red[wt * kMaxT + t] = vals[t];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t < T) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) s += red[w * kMaxT + t];
        vals[t] = s;
      }
    }
  }
}

// Surrogate derivative for the training kernels (gradients are compared within a
// tolerance, so the fast-division intrinsic is used; the LIF backward entry point in
// lif.cu keeps IEEE division for bit-exact parity with the reference).
__device__ __forceinline__ float surrogate_grad(int kind, float u, float k, float c) {
  if (kind == SPK_SURROGATE_SUPERSPIKE) {
    const float a = fmaf(k, fabsf(u), 1.0f);
    return __fdividef(1.0f, a * a);
  }
  const float z = c * u;
  return __fdividef(0.5f * k, fmaf(z, z, 1.0f));
}

// NW warps per token: NW = 1 -> each of the 4 warps of a block handles its own tokens;
// NW = 4 -> the whole block handles one token at a time.
template <int NW, int V, int CM>
__global__ void __launch_bounds__(kThreads) ln_lif_fwd_kernel(const FwdParams p) {
  __shared__ float red[4 * kMaxT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wt = NW == 1 ? 0 : warp;                  // warp index within the token
  const int slots = kThreads / 32 / NW;               // tokens per block at a time
  const int slot = NW == 1 ? warp : 0;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const int T = p.T, D = p.D, cpt = p.cpt;
  float g[CM], bl[CM];
#pragma unroll
  for (int i = 0; i < CM; ++i) {
    const int c = col_of<NW, V>(i, wt, lane);
    g[i] = (i < cpt && p.gamma) ? __ldg(p.gamma + c) : 1.0f;
    bl[i] = (i < cpt && p.beta_ln) ? __ldg(p.beta_ln + c) : 0.0f;
  }
  for (int64_t tok = (int64_t)blockIdx.x * slots + slot; tok < p.R; tok += (int64_t)gridDim.x * slots) {
    float x[kMaxT][CM];
    float s1[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      s1[t] = 0.0f;
      if (t < T) {
        const int64_t rb = ((int64_t)t * p.R + tok) * D;
#pragma unroll
        for (int i = 0; i < CM; i += V) {
          if (i < cpt) {
            if constexpr (V == 4) {
              load4(p.pre, p.pre_dtype, rb + col_of<NW, V>(i, wt, lane), &x[t][i]);
            } else {
              x[t][i] = load_elem(p.pre, p.pre_dtype, rb + col_of<NW, V>(i, wt, lane));
            }
          } else {
#pragma unroll
            for (int v = 0; v < V; ++v) x[t][i + v] = 0.0f;
          }
        }
#pragma unroll
        for (int i = 0; i < CM; ++i) s1[t] += x[t][i];
      }
    }
    token_sums<NW>(s1, T, red, wt);
    float mean[kMaxT], s2[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      mean[t] = s1[t] / (float)D;
      s2[t] = 0.0f;
      if (t < T) {
#pragma unroll
        for (int i = 0; i < CM; ++i) {
          if (i < cpt) {
            const float d = x[t][i] - mean[t];
            s2[t] = fmaf(d, d, s2[t]);
          }
        }
      }
    }
    token_sums<NW>(s2, T, red, wt);
    float rstd[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      rstd[t] = 1.0f / sqrtf(s2[t] / (float)D + p.eps);
      if (t < T && wt == 0 && lane == 0) p.stats[(int64_t)t * p.R + tok] = make_float2(mean[t], rstd[t]);
    }
    // LIF over t; the spikes overwrite x in place, then leave in vectors
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i >= cpt) continue;
      float v = 0.0f;
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
        const float y = fmaf((x[t][i] - mean[t]) * rstd[t], g[i], bl[i]);
        const float cur = p.gain != 1.0f ? __fmul_rn(y, p.gain) : y;
        v = __fadd_rn(__fmul_rn(v, lb), cur);
        const bool s = v > vth;
        x[t][i] = s ? 1.0f : 0.0f;
        v = s ? vr : v;
      }
    }
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const int64_t rb = ((int64_t)t * p.R + tok) * D;
#pragma unroll
      for (int i = 0; i < CM; i += V) {
        if (i >= cpt) continue;
        if constexpr (V == 4)
          store4(p.spikes, p.spike_dtype, rb + col_of<NW, V>(i, wt, lane), &x[t][i]);
        else
          store_elem(p.spikes, p.spike_dtype, rb + col_of<NW, V>(i, wt, lane), x[t][i]);
      }
    }
  }
}

template <int NW, int V, int CM>
__global__ void __launch_bounds__(kThreads) ln_lif_bwd_kernel(const BwdParams p) {
  __shared__ float red[4 * kMaxT];
  __shared__ float blk[4][kMaxCpt * 32 * 2 + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wt = NW == 1 ? 0 : warp;
  const int slots = kThreads / 32 / NW;
  const int slot = NW == 1 ? warp : 0;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const int T = p.T, D = p.D, cpt = p.cpt;
  const float invD = 1.0f / (float)D;
  float g[CM], bl[CM], acc_g[CM], acc_b[CM];
#pragma unroll
  for (int i = 0; i < CM; ++i) {
    const int c = col_of<NW, V>(i, wt, lane);
    g[i] = (i < cpt && p.gamma) ? __ldg(p.gamma + c) : 1.0f;
    bl[i] = (i < cpt && p.beta_ln) ? __ldg(p.beta_ln + c) : 0.0f;
    acc_g[i] = 0.0f;
    acc_b[i] = 0.0f;
  }
  float acc_lb = 0.0f;
  for (int64_t tok = (int64_t)blockIdx.x * slots + slot; tok < p.R; tok += (int64_t)gridDim.x * slots) {
    float xh[kMaxT][CM], gy[kMaxT][CM];
    float rstd[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      rstd[t] = 0.0f;
      if (t < T) {
        const float2 st = p.stats[(int64_t)t * p.R + tok];
        rstd[t] = st.y;
        const int64_t rb = ((int64_t)t * p.R + tok) * D;
#pragma unroll
        for (int i = 0; i < CM; i += V) {
          if (i < cpt) {
            const int64_t e = rb + col_of<NW, V>(i, wt, lane);
            if constexpr (V == 4) {
              load4(p.pre, p.pre_dtype, e, &xh[t][i]);
              load4(p.g_spikes, p.gs_dtype, e, &gy[t][i]);
            } else {
              xh[t][i] = load_elem(p.pre, p.pre_dtype, e);
              gy[t][i] = load_elem(p.g_spikes, p.gs_dtype, e);
            }
#pragma unroll
            for (int v = 0; v < V; ++v) xh[t][i + v] = (xh[t][i + v] - st.x) * st.y;
          } else {
#pragma unroll
            for (int v = 0; v < V; ++v) {
              xh[t][i + v] = 0.0f;
              gy[t][i + v] = 0.0f;
            }
          }
        }
      }
    }
    // LIF: recompute the pre-reset membrane, then BPTT (gy: dL/ds -> dL/dy)
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i >= cpt) continue;
      float u[kMaxT];
      bool sp[kMaxT];
      float v = 0.0f;
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
        const float y = fmaf(xh[t][i], g[i], bl[i]);
        const float cur = p.gain != 1.0f ? __fmul_rn(y, p.gain) : y;
        v = __fadd_rn(__fmul_rn(v, lb), cur);
        u[t] = v;
        sp[t] = v > vth;
        v = sp[t] ? vr : v;
      }
      float gstate = 0.0f;
#pragma unroll
      for (int t = kMaxT - 1; t >= 0; --t) {
        if (t >= T) continue;
        const float sg = surrogate_grad(p.surrogate, u[t] - vth, p.k, p.c_arctan);
        const float gv = gy[t][i] * sg + (sp[t] ? 0.0f : gstate);
        const float vprev = t > 0 ? (sp[t - 1] ? vr : u[t - 1]) : 0.0f;
        acc_lb = fmaf(gv, vprev, acc_lb);
        gstate = gv * lb;
        gy[t][i] = p.gain != 1.0f ? gv * p.gain : gv;  // dL/dy
      }
    }
    // LayerNorm backward per row
    float a[kMaxT], b[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      a[t] = 0.0f;
      b[t] = 0.0f;
      if (t < T) {
#pragma unroll
        for (int i = 0; i < CM; ++i) {
          if (i < cpt) {
            const float gx = gy[t][i] * g[i];
            a[t] += gx;
            b[t] = fmaf(gx, xh[t][i], b[t]);
            acc_g[i] = fmaf(gy[t][i], xh[t][i], acc_g[i]);
            acc_b[i] += gy[t][i];
          }
        }
      }
    }
    token_sums<NW>(a, T, red, wt);
    token_sums<NW>(b, T, red, wt);
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const float ma = a[t] * invD, mb = b[t] * invD;
      const int64_t rb = ((int64_t)t * p.R + tok) * D;
#pragma unroll
      for (int i = 0; i < CM; ++i) gy[t][i] = rstd[t] * (gy[t][i] * g[i] - ma - xh[t][i] * mb);
#pragma unroll
      for (int i = 0; i < CM; i += V) {
        if (i >= cpt) continue;
        if constexpr (V == 4)
          store4(p.g_pre, p.pre_dtype, rb + col_of<NW, V>(i, wt, lane), &gy[t][i]);
        else
          store_elem(p.g_pre, p.pre_dtype, rb + col_of<NW, V>(i, wt, lane), gy[t][i]);
      }
    }
  }
  // per-block partials: the warps of a block own the same columns when NW = 1, so they are
  // combined in warp order first; NW = 4 warps own disjoint columns
  const int W = 2 * D + 1;
  float* out = p.part + (int64_t)blockIdx.x * W;
  if constexpr (NW == 1) {
    // (for NW = 1 the D <= 512 columns index blk directly)
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i < cpt) {
        const int c = col_of<NW, V>(i, 0, lane);
        blk[warp][c] = acc_g[i];
        blk[warp][kMaxCpt * 32 + c] = acc_b[i];
      }
    }
    const float lbw = warp_sum(acc_lb);
    if (lane == 0) blk[warp][kMaxCpt * 32 * 2] = lbw;
    __syncthreads();
    if (warp == 0) {
      for (int c = lane; c < D; c += 32) {
        out[c] = ((blk[0][c] + blk[1][c]) + blk[2][c]) + blk[3][c];
        out[D + c] = ((blk[0][kMaxCpt * 32 + c] + blk[1][kMaxCpt * 32 + c]) + blk[2][kMaxCpt * 32 + c]) +
                     blk[3][kMaxCpt * 32 + c];
      }
      if (lane == 0)
        out[2 * D] = ((blk[0][kMaxCpt * 64] + blk[1][kMaxCpt * 64]) + blk[2][kMaxCpt * 64]) + blk[3][kMaxCpt * 64];
    }
  } else {
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i < cpt) {
        const int c = col_of<NW, V>(i, wt, lane);
        out[c] = acc_g[i];
        out[D + c] = acc_b[i];
      }
    }
    const float lbw = warp_sum(acc_lb);
    if (lane == 0) red[warp] = lbw;
    __syncthreads();
    if (threadIdx.x == 0) out[2 * D] = ((red[0] + red[1]) + red[2]) + red[3];
  }
}

// column c of the [rows][W] partials (dgamma, dbeta, LIF beta): 8 row groups
// (rows r = g mod 8, in order) per column, combined in group order
__global__ void __launch_bounds__(256) sum_columns_kernel(const float* __restrict__ part, int rows, int W,
                                                          float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                          float* __restrict__ dlif_beta, int D) {
  __shared__ float acc[8][33];
  const int cl = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  float s = 0.0f;
  if (c < W)
    for (int r = grp; r < rows; r += 8) s += part[(int64_t)r * W + c];
  acc[grp][cl] = s;
  __syncthreads();
  if (grp != 0 || c >= W) return;
  s = acc[0][cl];
#pragma unroll
  for (int g = 1; g < 8; ++g) s += acc[g][cl];
  if (c < D) {
    if (dgamma) dgamma[c] = s;
  } else if (c < 2 * D) {
    if (dbeta) dbeta[c - D] = s;
  } else if (dlif_beta) {
    *dlif_beta = s;
  }
}

inline int pick_nw(int D) { return D <= 32 * kMaxCpt ? 1 : 4; }

// blocks_per_sm: 2 for the backward (persistent: it keeps per-block partial sums, and its
// register use allows two blocks per SM), 8 for the forward
inline int grid_blocks(int64_t R, int nw, int blocks_per_sm = 2) {
  const int64_t slots = 4 / nw;
  int64_t need = (R + slots - 1) / slots;
  const int64_t cap = (int64_t)num_sms() * blocks_per_sm;
  if (need > cap) need = cap;
  return need < 1 ? 1 : (int)need;
}

}  // namespace lnlif

using namespace lnlif;

static int check_ln_lif(int T, int64_t R, int D) {
  SPK_REQUIRE(T >= 1 && T <= kMaxT, SPK_ERR_SHAPE, "T=%d outside [1, %d]", T, kMaxT);
  SPK_REQUIRE(R >= 0, SPK_ERR_SHAPE, "R negative");
  SPK_REQUIRE(D >= 32 && D % 32 == 0 && D <= 4 * 32 * kMaxCpt && (D <= 32 * kMaxCpt || D % 128 == 0), SPK_ERR_SHAPE,
              "D=%d unsupported (multiple of 32 up to %d, multiple of 128 above %d)", D, 4 * 32 * kMaxCpt,
              32 * kMaxCpt);
  return SPK_OK;
}

}  // namespace spk

extern "C" {

int64_t spk_ln_lif_bwd_workspace_bytes(int64_t T, int64_t R, int64_t D) {
  (void)T;
  const int nw = spk::lnlif::pick_nw((int)D);
  const int64_t slots = 4 / nw;
  int64_t need = (R + slots - 1) / slots;
  const int64_t cap = 296ll * 2;  // upper bound of the grid on any sm_100 part with up to 296 SMs
  if (need > cap) need = cap;
  if (need < 1) need = 1;
  return need * (2 * D + 1) * (int64_t)sizeof(float);
}

int spk_ln_lif_fwd(const void* pre, int pre_dtype, const float* ln_gamma, const float* ln_beta, float ln_eps,
                   const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain, int64_t T,
                   int64_t R, int64_t D, void* spikes, int spike_dtype, float* stats, void* stream) {
  using namespace spk;
  int rc = check_ln_lif((int)T, R, (int)D);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE((pre && spikes && stats) || R == 0, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID, "null LIF parameter");
  SPK_REQUIRE(pre_dtype == SPK_F32 || pre_dtype == SPK_F16 || pre_dtype == SPK_BF16, SPK_ERR_INVALID,
              "pre dtype %d not supported", pre_dtype);
  SPK_REQUIRE(spike_dtype >= SPK_F32 && spike_dtype <= SPK_U8, SPK_ERR_INVALID, "spike dtype %d", spike_dtype);
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  if (R == 0) return SPK_OK;
  FwdParams p = {pre, pre_dtype, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vreset, in_gain, spikes,
                 spike_dtype, reinterpret_cast<float2*>(stats), (int)T, R, (int)D, 0};
  const int nw = pick_nw((int)D);
  p.cpt = (int)D / (32 * nw);
  const int grid = grid_blocks(R, nw, 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // exact-size register arrays for 12 columns per thread (D = 384, 1536), else up to 16
  if (p.cpt == 12)
    nw == 1 ? ln_lif_fwd_kernel<1, 4, 12><<<grid, kThreads, 0, st>>>(p)
            : ln_lif_fwd_kernel<4, 4, 12><<<grid, kThreads, 0, st>>>(p);
  else if (p.cpt % 4 == 0)
    nw == 1 ? ln_lif_fwd_kernel<1, 4, kMaxCpt><<<grid, kThreads, 0, st>>>(p)
            : ln_lif_fwd_kernel<4, 4, kMaxCpt><<<grid, kThreads, 0, st>>>(p);
  else
    nw == 1 ? ln_lif_fwd_kernel<1, 1, kMaxCpt><<<grid, kThreads, 0, st>>>(p)
            : ln_lif_fwd_kernel<4, 1, kMaxCpt><<<grid, kThreads, 0, st>>>(p);
  return check_launch("ln_lif_fwd_kernel");
}

int spk_ln_lif_bwd(const void* g_spikes, int gs_dtype, const void* pre, int pre_dtype, const float* stats,
                   const float* ln_gamma, const float* ln_beta, const float* lif_beta, const float* lif_vth,
                   const float* lif_vreset, float in_gain, int surrogate, float surrogate_k, int64_t T, int64_t R,
                   int64_t D, void* g_pre, float* g_gamma, float* g_beta_ln, float* g_lif_beta, void* workspace,
                   int64_t workspace_bytes, void* stream) {
  using namespace spk;
  int rc = check_ln_lif((int)T, R, (int)D);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE((g_spikes && pre && stats && g_pre) || R == 0, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID, "null LIF parameter");
  SPK_REQUIRE(pre_dtype == SPK_F32 || pre_dtype == SPK_F16 || pre_dtype == SPK_BF16, SPK_ERR_INVALID,
              "pre dtype %d not supported", pre_dtype);
  SPK_REQUIRE(gs_dtype == SPK_F32 || gs_dtype == SPK_F16 || gs_dtype == SPK_BF16, SPK_ERR_INVALID,
              "gradient dtype %d not supported", gs_dtype);
  SPK_REQUIRE(surrogate == SPK_SURROGATE_SUPERSPIKE || surrogate == SPK_SURROGATE_ARCTAN, SPK_ERR_INVALID,
              "unknown surrogate %d", surrogate);
  const int64_t need = spk_ln_lif_bwd_workspace_bytes(T, R, D);
  SPK_REQUIRE(workspace && workspace_bytes >= need, SPK_ERR_INVALID,
              "workspace of %lld bytes is smaller than spk_ln_lif_bwd_workspace_bytes() = %lld",
              (long long)workspace_bytes, (long long)need);
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int nw = pick_nw((int)D);
  const int grid = R == 0 ? 1 : grid_blocks(R, nw);
  SPK_REQUIRE((int64_t)grid * (2 * D + 1) * 4 <= workspace_bytes, SPK_ERR_INVALID, "workspace too small for %d blocks",
              grid);
  float* part = reinterpret_cast<float*>(workspace);
  if (R == 0) {
    cudaError_t e = cudaMemsetAsync(part, 0, (size_t)(2 * D + 1) * 4, st);
    if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  } else {
    BwdParams p = {g_spikes, gs_dtype, pre, pre_dtype, reinterpret_cast<const float2*>(stats), ln_gamma, ln_beta,
                   lif_beta, lif_vth, lif_vreset, in_gain, surrogate, surrogate_k,
                   (float)(3.14159265358979323846 / 2.0 * (double)surrogate_k), g_pre, part, (int)T, R, (int)D, 0};
    p.cpt = (int)D / (32 * nw);
    if (p.cpt == 12)
      nw == 1 ? ln_lif_bwd_kernel<1, 4, 12><<<grid, kThreads, 0, st>>>(p)
              : ln_lif_bwd_kernel<4, 4, 12><<<grid, kThreads, 0, st>>>(p);
    else if (p.cpt % 4 == 0)
      nw == 1 ? ln_lif_bwd_kernel<1, 4, kMaxCpt><<<grid, kThreads, 0, st>>>(p)
              : ln_lif_bwd_kernel<4, 4, kMaxCpt><<<grid, kThreads, 0, st>>>(p);
    else
      nw == 1 ? ln_lif_bwd_kernel<1, 1, kMaxCpt><<<grid, kThreads, 0, st>>>(p)
              : ln_lif_bwd_kernel<4, 1, kMaxCpt><<<grid, kThreads, 0, st>>>(p);
    if ((rc = check_launch("ln_lif_bwd_kernel")) != SPK_OK) return rc;
  }
  const int W = 2 * (int)D + 1;
  sum_columns_kernel<<<(W + 31) / 32, 256, 0, st>>>(part, grid, W, g_gamma, g_beta_ln, g_lif_beta, (int)D);
  return check_launch("sum_columns_kernel");
}

}  // extern "C"
