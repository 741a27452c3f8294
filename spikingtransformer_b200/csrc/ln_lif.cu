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
// The Linear's bias may be handed to these kernels instead of the GEMM: the
// forward adds it to pre before the LayerNorm, and the backward returns its
// gradient (the column sums of g_pre), so the library GEMM runs without a
// bias and no separate bias-gradient reduction is needed.
//
// Forward, per token: mean and variance by two passes, y = (x - mean) rstd
// gamma + beta, then the LIF over t with v = beta v + gain y (separately
// rounded multiply and add, as the reference), s = v > v_th,
// v = s ? v_reset : v.  Spikes are written and (mean, rstd) of every row is
// saved.  When D is a multiple of 128 one block handles one token (D/128
// warps, four consecutive columns per lane, the T rows kept as packed raw
// vectors and processed in t order); otherwise one warp handles one token
// with single interleaved columns.
//
// Backward, per token: x^ and the membrane are recomputed from the saved
// statistics; BPTT over t with the surrogate (SuperSpike or arctan) gives
// dL/dy; then the LayerNorm input gradient
//   dx = rstd (g - mean(g) - x^ mean(g x^)),  g = gamma dL/dy
// and per-column partial sums of dL/dgamma = sum dL/dy x^, dL/dbeta = sum
// dL/dy and dL/dbias = sum dx, plus the LIF beta gradient sum g_v v_prev, are
// kept per block and reduced in a fixed order by a second kernel.
#include <initializer_list>

#include "common.cuh"

namespace spk {
namespace lnlif {

constexpr int kThreads = 128;  // 4 warps
constexpr int kMaxCpt = 16;    // columns per thread
constexpr int kMaxT = 4;

struct FwdParams {
  const void* pre;
  int pre_dtype;
  const float* bias;  // [D] added to pre, or null
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
  int hd, seq;  // head-major spikes [T*B][D/hd][seq][hd] when hd > 0 (R = B * seq)
  int64_t ld;   // row stride of pre (and g_pre) in elements (D, or wider for a column slice)
  const float* residual;  // token-group kernels: spikes = residual + LIF output (fp32, row-major), or null
  __nv_bfloat16* out_bf16;  // with a residual: also a bf16 copy of the fp32 output, or null
};

struct BwdParams {
  const void* g_spikes;
  int gs_dtype;
  const void* pre;
  int pre_dtype;
  const float* bias;  // [D] added to pre, or null
  const float2* stats;
  const float* gamma;
  const float* beta_ln;
  const float *lif_beta, *lif_vth, *lif_vr;
  float gain;
  int surrogate;
  float k, c_arctan;
  void* g_pre;  // same dtype as pre
  float* part;  // [grid][3 D + 1]: dgamma, dbeta, dbias partials, LIF beta partial
  int T;
  int64_t R;
  int D, cpt;
  int hd, seq;  // head-major spikes [T*B][D/hd][seq][hd] when hd > 0 (R = B * seq)
  int64_t ld;   // row stride of pre (and g_pre) in elements (D, or wider for a column slice)
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

// four consecutive elements kept packed until their row is processed
template <int EB>
struct RawVec;
template <>
struct RawVec<2> {
  uint2 w;
};
template <>
struct RawVec<4> {
  float4 w;
};

template <int EB>
__device__ __forceinline__ void raw_load(RawVec<EB>& r, const void* p, int64_t i) {
  if constexpr (EB == 2)
    r.w = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
  else
    r.w = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
}

template <int EB>
__device__ __forceinline__ void raw_unpack(const RawVec<EB>& r, int dt, float* o) {
  if constexpr (EB == 4) {
    o[0] = r.w.x; o[1] = r.w.y; o[2] = r.w.z; o[3] = r.w.w;
  } else if (dt == SPK_F16) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.w.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  } else {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.w.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.w.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
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
  float g[CM], bl[CM], pb[CM];
#pragma unroll
  for (int i = 0; i < CM; ++i) {
    const int c = col_of<NW, V>(i, wt, lane);
    g[i] = (i < cpt && p.gamma) ? __ldg(p.gamma + c) : 1.0f;
    bl[i] = (i < cpt && p.beta_ln) ? __ldg(p.beta_ln + c) : 0.0f;
    pb[i] = (i < cpt && p.bias) ? __ldg(p.bias + c) : 0.0f;
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
        for (int i = 0; i < CM; ++i) x[t][i] += pb[i];
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
  __shared__ float blk[4][kMaxCpt * 32 * 3 + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wt = NW == 1 ? 0 : warp;
  const int slots = kThreads / 32 / NW;
  const int slot = NW == 1 ? warp : 0;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const int T = p.T, D = p.D, cpt = p.cpt;
  const float invD = 1.0f / (float)D;
  float g[CM], bl[CM], pb[CM], acc_g[CM], acc_b[CM], acc_d[CM];
#pragma unroll
  for (int i = 0; i < CM; ++i) {
    const int c = col_of<NW, V>(i, wt, lane);
    g[i] = (i < cpt && p.gamma) ? __ldg(p.gamma + c) : 1.0f;
    bl[i] = (i < cpt && p.beta_ln) ? __ldg(p.beta_ln + c) : 0.0f;
    pb[i] = (i < cpt && p.bias) ? __ldg(p.bias + c) : 0.0f;
    acc_g[i] = 0.0f;
    acc_b[i] = 0.0f;
    acc_d[i] = 0.0f;
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
            for (int v = 0; v < V; ++v) xh[t][i + v] = ((xh[t][i + v] + pb[i + v]) - st.x) * st.y;
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
      for (int i = 0; i < CM; ++i) {
        gy[t][i] = rstd[t] * (gy[t][i] * g[i] - ma - xh[t][i] * mb);
        if (i < cpt) acc_d[i] += gy[t][i];
      }
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
  const int W = 3 * D + 1;
  float* out = p.part + (int64_t)blockIdx.x * W;
  if constexpr (NW == 1) {
    // (for NW = 1 the D <= 512 columns index blk directly)
    constexpr int S = kMaxCpt * 32;
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i < cpt) {
        const int c = col_of<NW, V>(i, 0, lane);
        blk[warp][c] = acc_g[i];
        blk[warp][S + c] = acc_b[i];
        blk[warp][2 * S + c] = acc_d[i];
      }
    }
    const float lbw = warp_sum(acc_lb);
    if (lane == 0) blk[warp][3 * S] = lbw;
    __syncthreads();
    if (warp == 0) {
      for (int c = lane; c < D; c += 32) {
#pragma unroll
        for (int k = 0; k < 3; ++k)
          out[k * D + c] = ((blk[0][k * S + c] + blk[1][k * S + c]) + blk[2][k * S + c]) + blk[3][k * S + c];
      }
      if (lane == 0) out[3 * D] = ((blk[0][3 * S] + blk[1][3 * S]) + blk[2][3 * S]) + blk[3][3 * S];
    }
  } else {
#pragma unroll
    for (int i = 0; i < CM; ++i) {
      if (i < cpt) {
        const int c = col_of<NW, V>(i, wt, lane);
        out[c] = acc_g[i];
        out[D + c] = acc_b[i];
        out[2 * D + c] = acc_d[i];
      }
    }
    const float lbw = warp_sum(acc_lb);
    if (lane == 0) red[warp] = lbw;
    __syncthreads();
    if (threadIdx.x == 0) out[3 * D] = ((red[0] + red[1]) + red[2]) + red[3];
  }
}

// Offsets of a lane's four columns c in the spikes / their gradient: row-major
// [T*R][D], or head-major [T*B][D/hd][seq][hd] for attention (token r = b*seq
// + n, column c = h*hd + d), the layout the attention products read.
// Row (t, r) starts at t * t_stride + tok_off(r); the lane adds col_off.
struct SpikeLayout {
  int64_t t_stride;  // elements between step t and t + 1 of one token
  int64_t col_off;   // the lane's column offset within a token row
  int hd, seq;
  int64_t head_block;  // seq * hd
  __device__ __forceinline__ SpikeLayout(int64_t R, int D, int c, int hd_, int seq_) : hd(hd_), seq(seq_) {
    t_stride = R * D;  // both layouts: [T][R*D] with B = R / seq
    if (hd <= 0) {
      col_off = c;
      head_block = 0;
    } else {
      const int h = c / hd;
      head_block = (int64_t)seq * hd;
      col_off = h * head_block + (c - h * hd);
    }
  }
  __device__ __forceinline__ int64_t tok_off(int64_t tok, int D) const {
    if (hd <= 0) return tok * D;
    const int ti = (int)tok;  // R < 2^31 in this layout
    const int b = ti / seq, n = ti - b * seq;  // one 32-bit division per token
    return (int64_t)b * D * seq + (int64_t)n * hd;
  }
};

// ---------------------------------------------------------------------------
// One token per block (D % 128 == 0): NW = D / 128 warps, four consecutive
// columns per lane, so one 8- or 16-byte vector per row and lane.  The
// working set is a few dozen registers, and many blocks are resident per SM
// to keep enough loads in flight.  Row sums over the block go through
// double-buffered shared slots: one barrier per sum (a slot is rewritten only
// two sums later, after a barrier that every reader has passed).

constexpr int kTokMaxWarps = 16;  // D <= 2048
constexpr int kTokPfWarps = 12;   // the prefetching backward: D <= 1536 (fits 170 registers)

struct BlockSum {
  float2* red;  // [2][kTokMaxWarps]
  int buf;
  __device__ __forceinline__ float2 sum2(float2 v, int nw) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    float2* r = red + buf * kTokMaxWarps;
    if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
    __syncthreads();
    float2 s = make_float2(0.0f, 0.0f);
    for (int w = 0; w < nw; ++w) {
      s.x += r[w].x;
      s.y += r[w].y;
    }
    buf ^= 1;
    return s;
  }
  __device__ __forceinline__ float sum(float v, int nw) { return sum2(make_float2(v, 0.0f), nw).x; }
};

// Mean and sum of squared deviations of a row in one block reduction: each
// lane starts from its four columns, and partial (mean, M2) pairs are merged
// with the parallel-variance formula (Chan et al.), in a fixed order, so
// every thread gets the same result.  Within a warp both partners of a
// shuffle hold equal counts: mean = (ma + mb) / 2, M2 = M2a + M2b + d^2 n / 2.
__constant__ float2 c_merge_w[kTokMaxWarps] = {
    {0.f, 0.f},           {1.f / 2, 64.f},        {1.f / 3, 256.f / 3},   {1.f / 4, 96.f},
    {1.f / 5, 512.f / 5}, {1.f / 6, 640.f / 6},   {1.f / 7, 768.f / 7},   {1.f / 8, 112.f},
    {1.f / 9, 1024.f / 9}, {1.f / 10, 115.2f},    {1.f / 11, 1280.f / 11}, {1.f / 12, 1408.f / 12},
    {1.f / 13, 1536.f / 13}, {1.f / 14, 1664.f / 14}, {1.f / 15, 1792.f / 15}, {1.f / 16, 120.f}};

__device__ __forceinline__ float2 block_mean_m2(BlockSum& bs, float2 mm, int nw) {
  float n = 4.0f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mm.x, o);
    const float o2 = __shfl_xor_sync(0xffffffffu, mm.y, o);
    const float d = om - mm.x;
    mm.y = (mm.y + o2) + d * d * (0.5f * n);
    mm.x = 0.5f * (mm.x + om);
    n *= 2.0f;
  }
  if (nw == 1) return mm;
  float2* r = bs.red + bs.buf * kTokMaxWarps;
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = mm;
  __syncthreads();
  // merging warp w (128 values) into the first w warps: weights 1/(w+1) and
  // 128 w/(w+1), from a table
  float2 acc = r[0];
  for (int w = 1; w < nw; ++w) {
    const float2 b = r[w];
    const float d = b.x - acc.x;
    acc.x = fmaf(d, c_merge_w[w].x, acc.x);
    acc.y = fmaf(d * d, c_merge_w[w].y, acc.y + b.y);
  }
  bs.buf ^= 1;
  return acc;
}

// spikes of dtype SD (SPK_F32 / SPK_BF16 stored directly; -1: any dtype, chosen at run time)
template <int SD>
__device__ __forceinline__ void store_spikes4(void* p, int dt, int64_t i, const float* v) {
  if constexpr (SD == SPK_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (SD == SPK_BF16) {
    // 0/1 values: the bf16 bit patterns are 0x0000 / 0x3f80
    uint2 w;
    w.x = (v[0] != 0.0f ? 0x3f80u : 0u) | (v[1] != 0.0f ? 0x3f800000u : 0u);
    w.y = (v[2] != 0.0f ? 0x3f80u : 0u) | (v[3] != 0.0f ? 0x3f800000u : 0u);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) = w;
  } else {
    store4(p, dt, i, v);
  }
}

// Statistics: mean = sum * (1/D) and rstd = rsqrtf(var + eps) (within a few
// ulp of the IEEE divide and square root; the per-row division and square
// root dominated the instruction count of this kernel).
template <int EB, int SD>
__global__ void __launch_bounds__(32 * kTokMaxWarps) ln_lif_fwd_tok_kernel(const FwdParams p) {
  __shared__ float2 red[2 * kTokMaxWarps];
  BlockSum bs{red, 0};
  const int nw = blockDim.x >> 5;
  const int c = threadIdx.x * 4;  // this lane's four columns
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const int T = p.T, D = p.D;
  const float invD = 1.0f / (float)D;
  const float4 g4 = p.gamma ? __ldg(reinterpret_cast<const float4*>(p.gamma + c)) : make_float4(1.f, 1.f, 1.f, 1.f);
  const float4 b4 = p.beta_ln ? __ldg(reinterpret_cast<const float4*>(p.beta_ln + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 p4 = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float2 gg2[2] = {make_float2(g4.x, g4.y), make_float2(g4.z, g4.w)};
  const float2 bb2[2] = {make_float2(b4.x, b4.y), make_float2(b4.z, b4.w)};
  const float2 pp2[2] = {make_float2(p4.x, p4.y), make_float2(p4.z, p4.w)};
  const float2 beta2 = make_float2(lb, lb), gain2 = make_float2(p.gain, p.gain);
  const SpikeLayout lay(p.R, D, c, p.hd, p.seq);
  // the next token's rows are loaded while this one is processed
  RawVec<EB> nxt[kMaxT];
  if ((int64_t)blockIdx.x < p.R) {
#pragma unroll
    for (int t = 0; t < kMaxT; ++t)
      if (t < T) raw_load<EB>(nxt[t], p.pre, ((int64_t)t * p.R + blockIdx.x) * p.ld + c);
  }
  for (int64_t tok = blockIdx.x; tok < p.R; tok += gridDim.x) {
    const int64_t so = lay.tok_off(tok, D) + lay.col_off;
    RawVec<EB> raw[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) raw[t] = nxt[t];
    const int64_t tn = tok + gridDim.x;
    if (tn < p.R) {
#pragma unroll
      for (int t = 0; t < kMaxT; ++t)
        if (t < T) raw_load<EB>(nxt[t], p.pre, ((int64_t)t * p.R + tn) * p.ld + c);
    }
    float2 v2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      float x[4];
      raw_unpack<EB>(raw[t], p.pre_dtype, x);
      const float2 x01 = add2(make_float2(x[0], x[1]), pp2[0]), x23 = add2(make_float2(x[2], x[3]), pp2[1]);
      // this lane's (mean, M2), then one block merge
      const float lm = ((x01.x + x01.y) + (x23.x + x23.y)) * 0.25f;
      const float2 d01 = add2(x01, make_float2(-lm, -lm)), d23 = add2(x23, make_float2(-lm, -lm));
      const float2 q = fma2(d01, d01, mul2(d23, d23));
      const float2 mv = block_mean_m2(bs, make_float2(lm, q.x + q.y), nw);
      const float mean = mv.x;
      const float rstd = rsqrtf(fmaf(mv.y, invD, p.eps));
      const int64_t row = (int64_t)t * p.R + tok;
      if (threadIdx.x == 0) p.stats[row] = make_float2(mean, rstd);
      const float2 nm2 = make_float2(-mean, -mean), r2 = make_float2(rstd, rstd);
      const float2 xs[2] = {x01, x23};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float2 y = fma2(mul2(add2(xs[j], nm2), r2), gg2[j], bb2[j]);
        const float2 cur = p.gain != 1.0f ? mul2(y, gain2) : y;
        const float2 u = add2(mul2(v2[j], beta2), cur);
        const bool sx = u.x > vth, sy = u.y > vth;
        x[2 * j] = sx ? 1.0f : 0.0f;
        x[2 * j + 1] = sy ? 1.0f : 0.0f;
        v2[j] = make_float2(sx ? vr : u.x, sy ? vr : u.y);
      }
      store_spikes4<SD>(p.spikes, p.spike_dtype, so + t * lay.t_stride, x);
    }
  }
}

// Backward, one token per block: the membrane is recomputed in t order from
// the saved statistics, then the steps are walked backwards; BPTT of step t
// gives dL/dy of row t, whose LayerNorm backward (one pair of block sums)
// runs at once.
template <int EBP, int EBG, bool PF, int SURR>
__global__ void __launch_bounds__(PF ? 32 * kTokPfWarps : 32 * kTokMaxWarps) ln_lif_bwd_tok_kernel(const BwdParams p) {
  __shared__ float2 red[2 * kTokMaxWarps];
  BlockSum bs{red, 0};
  const int nw = blockDim.x >> 5;
  const int c = threadIdx.x * 4;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const int T = p.T, D = p.D;
  const float invD = 1.0f / (float)D;
  const float4 g4 = p.gamma ? __ldg(reinterpret_cast<const float4*>(p.gamma + c)) : make_float4(1.f, 1.f, 1.f, 1.f);
  const float4 b4 = p.beta_ln ? __ldg(reinterpret_cast<const float4*>(p.beta_ln + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 p4 = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w}, pp[4] = {p4.x, p4.y, p4.z, p4.w};
  float2 acc_g2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float2 acc_b2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float2 acc_d2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float acc_lb = 0.0f;
  const SpikeLayout lay(p.R, D, c, p.hd, p.seq);
  RawVec<EBP> np_[kMaxT];
  RawVec<EBG> ng_[kMaxT];
  float2 ns_[kMaxT];
  auto load_tok = [&](int64_t tk, RawVec<EBP>* rp, RawVec<EBG>* rg, float2* st) {
    const int64_t so = lay.tok_off(tk, D) + lay.col_off;
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      st[t] = make_float2(0.0f, 1.0f);
      if (t >= T) continue;
      const int64_t row = (int64_t)t * p.R + tk;
      st[t] = p.stats[row];
      raw_load<EBP>(rp[t], p.pre, row * p.ld + c);
      raw_load<EBG>(rg[t], p.g_spikes, so + t * lay.t_stride);
    }
  };
  if (PF && (int64_t)blockIdx.x < p.R) load_tok(blockIdx.x, np_, ng_, ns_);
  for (int64_t tok = blockIdx.x; tok < p.R; tok += gridDim.x) {
    RawVec<EBP> rp[kMaxT];
    RawVec<EBG> rg[kMaxT];
    float2 st[kMaxT];
    if constexpr (PF) {
      // this token's rows were loaded during the previous one; start the next
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        rp[t] = np_[t];
        rg[t] = ng_[t];
        st[t] = ns_[t];
      }
      if (tok + gridDim.x < p.R) load_tok(tok + gridDim.x, np_, ng_, ns_);
    } else {
      load_tok(tok, rp, rg, st);
    }
    // membrane before reset at every step (pairs of columns in packed f32x2
    // arithmetic, each operation rounded like its scalar form)
    const float2 beta2 = make_float2(lb, lb), gain2 = make_float2(p.gain, p.gain);
    const float2 gg2[2] = {make_float2(gg[0], gg[1]), make_float2(gg[2], gg[3])};
    const float2 bb2[2] = {make_float2(bb[0], bb[1]), make_float2(bb[2], bb[3])};
    const float2 pp2[2] = {make_float2(pp[0], pp[1]), make_float2(pp[2], pp[3])};
    float2 u[kMaxT][2];
    {
      float2 v[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
        float x[4];
        raw_unpack<EBP>(rp[t], p.pre_dtype, x);
        const float2 m2 = make_float2(-st[t].x, -st[t].x), r2 = make_float2(st[t].y, st[t].y);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 xh = mul2(add2(add2(make_float2(x[2 * j], x[2 * j + 1]), pp2[j]), m2), r2);
          const float2 y = fma2(xh, gg2[j], bb2[j]);
          const float2 cur = p.gain != 1.0f ? mul2(y, gain2) : y;
          const float2 uu = add2(mul2(v[j], beta2), cur);
          u[t][j] = uu;
          v[j].x = uu.x > vth ? vr : uu.x;
          v[j].y = uu.y > vth ? vr : uu.y;
        }
      }
    }
    float2 gstate[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const float2 nvth2 = make_float2(-vth, -vth);
#pragma unroll
    for (int t = kMaxT - 1; t >= 0; --t) {
      if (t >= T) continue;
      float gyv[4], x[4];
      raw_unpack<EBG>(rg[t], p.gs_dtype, gyv);
      raw_unpack<EBP>(rp[t], p.pre_dtype, x);
      const float2 m2 = make_float2(-st[t].x, -st[t].x), r2 = make_float2(st[t].y, st[t].y);
      float2 gy[2], xh[2];
      float2 av = make_float2(0.f, 0.f), bv = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        // BPTT step t: dL/ds -> dL/dy
        const float2 d = add2(u[t][j], nvth2);
        float2 sg;
        if constexpr (SURR == SPK_SURROGATE_SUPERSPIKE) {
          const float2 q = fma2(make_float2(p.k, p.k), make_float2(fabsf(d.x), fabsf(d.y)), make_float2(1.f, 1.f));
          const float2 q2 = mul2(q, q);
          sg = make_float2(__fdividef(1.0f, q2.x), __fdividef(1.0f, q2.y));
        } else {
          const float2 z = mul2(make_float2(p.c_arctan, p.c_arctan), d);
          const float2 den = fma2(z, z, make_float2(1.f, 1.f));
          const float hk = 0.5f * p.k;
          sg = make_float2(__fdividef(hk, den.x), __fdividef(hk, den.y));
        }
        const bool sx = u[t][j].x > vth, sy = u[t][j].y > vth;
        const float2 from = make_float2(sx ? 0.0f : gstate[j].x, sy ? 0.0f : gstate[j].y);
        const float2 gv = fma2(make_float2(gyv[2 * j], gyv[2 * j + 1]), sg, from);
        float2 vprev = make_float2(0.f, 0.f);
        if (t > 0) {
          vprev.x = u[t - 1][j].x > vth ? vr : u[t - 1][j].x;
          vprev.y = u[t - 1][j].y > vth ? vr : u[t - 1][j].y;
        }
        const float2 lbp = mul2(gv, vprev);
        acc_lb += lbp.x + lbp.y;
        gstate[j] = mul2(gv, beta2);
        gy[j] = p.gain != 1.0f ? mul2(gv, gain2) : gv;
        // LayerNorm backward terms of row t
        xh[j] = mul2(add2(add2(make_float2(x[2 * j], x[2 * j + 1]), pp2[j]), m2), r2);
        const float2 gx = mul2(gy[j], gg2[j]);
        av = add2(av, gx);
        bv = fma2(gx, xh[j], bv);
        acc_g2[j] = fma2(gy[j], xh[j], acc_g2[j]);
        acc_b2[j] = add2(acc_b2[j], gy[j]);
      }
      const float2 ab = bs.sum2(make_float2(av.x + av.y, bv.x + bv.y), nw);
      const float2 ma = make_float2(-ab.x * invD, -ab.x * invD), mb = make_float2(-ab.y * invD, -ab.y * invD);
      float dx[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        // dx = rstd (g gamma - mean(g gamma) - x^ mean(g gamma x^))
        const float2 dd = mul2(fma2(xh[j], mb, fma2(gy[j], gg2[j], ma)), r2);
        dx[2 * j] = dd.x;
        dx[2 * j + 1] = dd.y;
        acc_d2[j] = add2(acc_d2[j], dd);
      }
      store4(p.g_pre, p.pre_dtype, ((int64_t)t * p.R + tok) * p.ld + c, dx);
    }
  }
  // per-block partials: each thread owns its four columns; the LIF beta term
  // is summed over the block.  Rows are 3 D + 1 floats long, so a row start is
  // only 4-byte aligned: scalar stores.
  float* out = p.part + (int64_t)blockIdx.x * (3 * D + 1);
  const float acc_g[4] = {acc_g2[0].x, acc_g2[0].y, acc_g2[1].x, acc_g2[1].y};
  const float acc_b[4] = {acc_b2[0].x, acc_b2[0].y, acc_b2[1].x, acc_b2[1].y};
  const float acc_d[4] = {acc_d2[0].x, acc_d2[0].y, acc_d2[1].x, acc_d2[1].y};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    out[c + e] = acc_g[e];
    out[D + c + e] = acc_b[e];
    out[2 * D + c + e] = acc_d[e];
  }
  const float lbs = bs.sum(acc_lb, nw);
  if (threadIdx.x == 0) out[3 * D] = lbs;
}

// ---------------------------------------------------------------------------
// One token per group of G warps, twelve columns per lane: D = 384 G with
// G = 1, 2 or 4 (the model's D = 384 and 1536).  A lane holds three 4-column
// vectors of every row, at columns 128 (i G + wg) + 4 lane (wg the warp's
// index in its group), so one warp access of vector i covers 128 consecutive
// columns.  The row reductions of a token run once for all T rows together
// (forward: each row's mean and M2; backward: each row's two LayerNorm sums):
// by shuffles within a warp and, for G > 1, through double-buffered shared
// slots behind a named barrier of the group.  The per-row costs (reductions,
// statistics, addressing) are spread over twelve elements per lane, and a
// single-warp token needs no barrier.

constexpr int kGrpWarps = 8;  // warps per block
constexpr int kGrpNV = 3;     // 4-column vectors per lane and row
constexpr int kGrpFwdStages = 2;  // staged tokens per warp: the rows of kStages - 1 tokens are in flight
constexpr int kGrpBwdStages = 2;
constexpr int kGrpBwdNV = 3;      // the backward's 4-column vectors per lane and row (1 or 3)

inline bool use_grp(int D) { return D == 384 || D == 768 || D == 1536; }

// Mean and M2 of up to kMaxT rows over the 32 lanes of a warp, each lane
// starting from n0 values; the partners of every shuffle hold equal counts,
// so mean = (ma + mb) / 2 and M2 = M2a + M2b + d^2 n / 2, and every lane ends
// with the same result.
__device__ __forceinline__ void warp_mean_m2(float2 (&mm)[kMaxT], int T, float n0) {
  float n = n0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const float om = __shfl_xor_sync(0xffffffffu, mm[t].x, o);
      const float o2 = __shfl_xor_sync(0xffffffffu, mm[t].y, o);
      const float d = om - mm[t].x;
      mm[t].y = (mm[t].y + o2) + d * d * (0.5f * n);
      mm[t].x = 0.5f * (mm[t].x + om);
    }
    n *= 2.0f;
  }
}

// sums of up to kMaxT float2 values over the 32 lanes of a warp (the same on every lane)
__device__ __forceinline__ void warp_sum2(float2 (&v)[kMaxT], int T) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      v[t].x += __shfl_xor_sync(0xffffffffu, v[t].x, o);
      v[t].y += __shfl_xor_sync(0xffffffffu, v[t].y, o);
    }
  }
}

// the value of row `lane` (lanes < kMaxT) of a per-row register array
__device__ __forceinline__ float2 row_of_lane(const float2 (&v)[kMaxT], int lane) {
  float2 r = v[0];
#pragma unroll
  for (int t = 1; t < kMaxT; ++t)
    if (lane == t) r = v[t];
  return r;
}

// Exchange of per-warp row values between the G warps of a token group:
// slot [buf][grp][w][t]; one named barrier (id 1 + grp) per exchange.  A slot
// is rewritten two exchanges later, after a barrier that every reader of it
// has passed.
template <int G, int W>
struct GroupXch {
  float2* slots;  // [2][NG][G][kMaxT]
  int grp, wg, buf;
  __device__ __forceinline__ float2* put(const float2 (&v)[kMaxT], int lane) {
    constexpr int NG = W / G;
    float2* base = slots + ((size_t)buf * NG + grp) * G * kMaxT;
    if (lane < kMaxT) base[wg * kMaxT + lane] = row_of_lane(v, lane);
    named_bar_sync(1 + grp, 32 * G);
    buf ^= 1;
    return base;
  }
  // (mean, M2) of every row merged over the group's warps in warp order; each
  // warp contributed n_w values per row
  __device__ __forceinline__ void merge_mean_m2(float2 (&mm)[kMaxT], int T, int lane, float n_w) {
    if constexpr (G > 1) {
      const float2* r = put(mm, lane);
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
        float2 acc = r[t];
#pragma unroll
        for (int w = 1; w < G; ++w) {
          // merging warp w into the first w warps: weights 1/(w+1) and n_w w/(w+1)
          const float2 b = r[w * kMaxT + t];
          const float d = b.x - acc.x;
          acc.x = fmaf(d, 1.0f / (float)(w + 1), acc.x);
          acc.y = fmaf(d * d, n_w * (float)w / (float)(w + 1), acc.y + b.y);
        }
        mm[t] = acc;
      }
    }
  }
  __device__ __forceinline__ void sum(float2 (&v)[kMaxT], int T, int lane) {
    if constexpr (G > 1) {
      const float2* r = put(v, lane);
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
        float2 acc = r[t];
#pragma unroll
        for (int w = 1; w < G; ++w) {
          acc.x += r[w * kMaxT + t].x;
          acc.y += r[w * kMaxT + t].y;
        }
        v[t] = acc;
      }
    }
  }
};

template <int EB>
__device__ __forceinline__ void cp_async_vec(RawVec<EB>* dst, const void* src) {
  if constexpr (EB == 2)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
  else
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Four consecutive fp32 values loaded afresh at every call (volatile: not
// hoisted out of the token loop and kept in registers for the whole kernel)
__device__ __forceinline__ float4 ld_fresh4(const float* q) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(q));
  return v;
}

// The LayerNorm parameters of the four columns c..c+3, as pairs: gamma and
// beta scaled by the LIF input gain (the LIF's input is gain (x^ gamma +
// beta), formed as x^ (gain gamma) + gain beta by the forward and by the
// backward's recomputation alike), and the Linear bias.
template <typename Params>
__device__ __forceinline__ void ln_params(const Params& p, int c, float2 gain2, float2 (&gq)[2], float2 (&bq)[2],
                                          float2 (&pq)[2]) {
  const float4 g4 = p.gamma ? ld_fresh4(p.gamma + c) : make_float4(1.f, 1.f, 1.f, 1.f);
  const float4 b4 = p.beta_ln ? ld_fresh4(p.beta_ln + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 p4 = p.bias ? ld_fresh4(p.bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  gq[0] = mul2(make_float2(g4.x, g4.y), gain2);
  gq[1] = mul2(make_float2(g4.z, g4.w), gain2);
  bq[0] = mul2(make_float2(b4.x, b4.y), gain2);
  bq[1] = mul2(make_float2(b4.z, b4.w), gain2);
  pq[0] = make_float2(p4.x, p4.y);
  pq[1] = make_float2(p4.z, p4.w);
}

// RESID: the output is residual + spikes in fp32 (row-major, the residual stream of a
// transformer layer, Encoder.py:19-22 / Decoder.py:18-24), with an optional bf16 copy.
template <int EB, int SD, int G, bool RESID = false>
__global__ void __launch_bounds__(32 * kGrpWarps, EB == 2 ? 2 : 1) ln_lif_fwd_grp_kernel(const FwdParams p) {
  constexpr int NV = kGrpNV, NG = kGrpWarps / G;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float2 xch[G > 1 ? 2 * NG * G * kMaxT : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / G, wg = warp - grp * G;
  constexpr int S = kGrpFwdStages;
  // this warp's S stages of [kMaxT][NV][32 lanes] pre-activation vectors
  RawVec<EB>* pre_s = reinterpret_cast<RawVec<EB>*>(smem) + (size_t)warp * S * kMaxT * NV * 32;
  auto pre_at = [&](int s, int t, int i) { return pre_s + ((s * kMaxT + t) * NV + i) * 32 + lane; };
  GroupXch<G, kGrpWarps> gx{xch, grp, wg, 0};
  const int T = p.T;
  const float invD = 1.0f / (float)p.D;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const SpikeLayout lay(p.R, p.D, 0, p.hd, p.seq);
  const float2 beta2 = make_float2(lb, lb), gain2 = make_float2(p.gain, p.gain);
  int cols[NV];
  int64_t coff[NV];
  float2 gg[NV][2], bb[NV][2], pb[NV][2];  // gain gamma, gain beta, bias
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 128 * (i * G + wg) + 4 * lane;
    cols[i] = c;
    coff[i] = SpikeLayout(p.R, p.D, c, p.hd, p.seq).col_off;
    ln_params(p, c, gain2, gg[i], bb[i], pb[i]);
  }
  const int64_t step = (int64_t)gridDim.x * NG;
  int64_t tok = (int64_t)blockIdx.x * NG + grp;
  // the rows of the next S - 1 tokens are in flight while this one is processed
  auto issue = [&](int64_t tk, int s) {
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const int64_t rb = ((int64_t)t * p.R + tk) * p.ld;
#pragma unroll
      for (int i = 0; i < NV; ++i)
        cp_async_vec<EB>(pre_at(s, t, i), reinterpret_cast<const unsigned char*>(p.pre) + (rb + cols[i]) * EB);
    }
  };
#pragma unroll
  for (int k = 0; k < S - 1; ++k) {
    if (tok + k * step < p.R) issue(tok + k * step, k);
    cp_async_commit();
  }
  int s = 0;
  for (; tok < p.R; tok += step, s = s + 1 == S ? 0 : s + 1) {
    const int64_t tn = tok + (S - 1) * step;
    if (tn < p.R) issue(tn, s == 0 ? S - 1 : s - 1);
    cp_async_commit();
    cp_async_wait<S - 1>();  // this token's vectors have landed
    // each row's (mean, M2): the lane's twelve values, then the warp, then the group
    float2 mm[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      mm[t] = make_float2(0.0f, 0.0f);
      if (t >= T) continue;
      float2 xs[NV][2];
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float x[4];
        raw_unpack<EB>(*pre_at(s, t, i), p.pre_dtype, x);
        xs[i][0] = add2(make_float2(x[0], x[1]), pb[i][0]);
        xs[i][1] = add2(make_float2(x[2], x[3]), pb[i][1]);
        sum += (xs[i][0].x + xs[i][0].y) + (xs[i][1].x + xs[i][1].y);
      }
      const float lm = sum * (1.0f / (4 * NV));
      const float2 nl = make_float2(-lm, -lm);
      float2 q = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 d = add2(xs[i][j], nl);
          q = fma2(d, d, q);
        }
      mm[t] = make_float2(lm, q.x + q.y);
    }
    warp_mean_m2(mm, T, (float)(4 * NV));
    gx.merge_mean_m2(mm, T, lane, (float)(32 * 4 * NV));
    float2 nm[kMaxT], rs[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      const float rstd = rsqrtf(fmaf(mm[t].y, invD, p.eps));
      nm[t] = make_float2(-mm[t].x, -mm[t].x);
      rs[t] = make_float2(rstd, rstd);
      mm[t].y = rstd;
    }
    if (wg == 0 && lane < T) p.stats[(int64_t)lane * p.R + tok] = row_of_lane(mm, lane);
    // LayerNorm output and the LIF over t
    const int64_t sb = lay.tok_off(tok, p.D);
    float2 v[NV][2];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i][0] = v[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float x[4];
        raw_unpack<EB>(*pre_at(s, t, i), p.pre_dtype, x);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 xb = add2(make_float2(x[2 * j], x[2 * j + 1]), pb[i][j]);
          const float2 u = add2(mul2(v[i][j], beta2), fma2(mul2(add2(xb, nm[t]), rs[t]), gg[i][j], bb[i][j]));
          const bool sx = u.x > vth, sy = u.y > vth;
          x[2 * j] = sx ? 1.0f : 0.0f;
          x[2 * j + 1] = sy ? 1.0f : 0.0f;
          v[i][j] = make_float2(sx ? vr : u.x, sy ? vr : u.y);
        }
        const int64_t oi = sb + t * lay.t_stride + coff[i];
        if constexpr (RESID) {
          // spike counts: the sum of a small integer and 0/1 is exact in fp32 and bf16
          const float4 r = __ldg(reinterpret_cast<const float4*>(p.residual + oi));
          const float4 o = make_float4(r.x + x[0], r.y + x[1], r.z + x[2], r.w + x[3]);
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.spikes) + oi) = o;
          if (p.out_bf16) {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y), hi = __floats2bfloat162_rn(o.z, o.w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&lo);
            w.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(p.out_bf16 + oi) = w;
          }
        } else {
          store_spikes4<SD>(p.spikes, p.spike_dtype, oi, x);
        }
      }
    }
  }
}

// Backward staging: per warp, a ring of stages, each [kMaxT][NV][32 lanes]
// vectors of the pre-activation, the same of the spike gradient, and the
// token's kMaxT row statistics.  Each lane copies (cp.async) and later reads
// only its own vectors, so a lane's wait_group is the only synchronisation
// the vectors need; the statistics, copied by lanes t < T, are read by every
// lane after a __syncwarp.
template <int EBP, int EBG, int NV>
constexpr size_t grp_bwd_stage_bytes() {
  return (size_t)kMaxT * NV * 32 * (4 * EBP + 4 * EBG) + kMaxT * sizeof(float2);
}
// fp32 pre-activation and gradient with three vectors per lane: one stage (two would exceed
// the shared memory)
template <int EBP, int EBG, int NV>
constexpr int grp_bwd_stages() {
  return NV == 3 && EBP + EBG > 6 ? 1 : kGrpBwdStages;
}
// warps per block: 8 with three vectors per lane (234 registers), 12 with one
template <int NV>
constexpr int grp_bwd_warps() {
  return NV == 3 ? 8 : 12;
}
// per warp: the stages, then the current token's x^ ([kMaxT][NV][32 lanes] float4)
template <int NV>
constexpr size_t grp_xhat_bytes() {
  return (size_t)kMaxT * NV * 32 * sizeof(float4);
}
template <int EBP, int EBG, int NV>
constexpr size_t grp_bwd_warp_bytes() {
  return grp_bwd_stages<EBP, EBG, NV>() * grp_bwd_stage_bytes<EBP, EBG, NV>() + grp_xhat_bytes<NV>();
}
template <int EBP, int EBG, int NV>
constexpr size_t grp_bwd_smem_bytes() {
  return (size_t)grp_bwd_warps<NV>() * grp_bwd_warp_bytes<EBP, EBG, NV>();
}

// Backward, one token per group: the token's rows arrive in shared memory one
// token ahead (cp.async); the membrane is recomputed in t order from the
// saved statistics; the steps are walked backwards (BPTT) giving dL/dy of
// every row, with the rows' two LayerNorm sums accumulated on the way; one
// reduction of those sums for all T rows; then dL/dx of every row.
template <int EBP, int EBG, int SURR, int NV, int G>
__global__ void __launch_bounds__(32 * grp_bwd_warps<NV>(), 1) ln_lif_bwd_grp_kernel(const BwdParams p) {
  constexpr int W = grp_bwd_warps<NV>(), NG = W / G;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float2 xch[G > 1 ? 2 * NG * G * kMaxT : 1];
  __shared__ float lb_red[W];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / G, wg = warp - grp * G;
  GroupXch<G, W> gx{xch, grp, wg, 0};
  const int T = p.T, D = p.D;
  const float invD = 1.0f / (float)D;
  const float lb = __ldg(p.lif_beta), vth = __ldg(p.lif_vth), vr = __ldg(p.lif_vr);
  const SpikeLayout lay(p.R, D, 0, p.hd, p.seq);
  constexpr int S = grp_bwd_stages<EBP, EBG, NV>();
  // this warp's stages (pre vectors, gradient vectors, row statistics), then x^
  RawVec<EBP>* pre_s = reinterpret_cast<RawVec<EBP>*>(smem + (size_t)warp * grp_bwd_warp_bytes<EBP, EBG, NV>());
  RawVec<EBG>* gs_s = reinterpret_cast<RawVec<EBG>*>(pre_s + S * kMaxT * NV * 32);
  float2* st_s = reinterpret_cast<float2*>(gs_s + S * kMaxT * NV * 32);
  float4* xh_s = reinterpret_cast<float4*>(st_s + S * kMaxT);
  auto xh_at = [&](int t, int i) { return xh_s + (t * NV + i) * 32 + lane; };
  auto pre_at = [&](int s, int t, int i) { return pre_s + ((s * kMaxT + t) * NV + i) * 32 + lane; };
  auto gs_at = [&](int s, int t, int i) { return gs_s + ((s * kMaxT + t) * NV + i) * 32 + lane; };
  const float2 beta2 = make_float2(lb, lb), gain2 = make_float2(p.gain, p.gain), nvth2 = make_float2(-vth, -vth);
  int cols[NV];
  int64_t coff[NV];
  float2 gg[NV][2], bb[NV][2], pb[NV][2];  // gain gamma, gain beta, bias
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 128 * (i * G + wg) + 4 * lane;
    cols[i] = c;
    coff[i] = SpikeLayout(p.R, D, c, p.hd, p.seq).col_off;
    ln_params(p, c, gain2, gg[i], bb[i], pb[i]);
  }
  float2 acc_g[NV][2], acc_b[NV][2], acc_d[NV][2];  // per column: sum of dL/dv x^, of dL/dv, of dL/dx
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc_g[i][j] = acc_b[i][j] = acc_d[i][j] = make_float2(0.0f, 0.0f);
  float2 acc_lb = make_float2(0.0f, 0.0f);
  const int64_t step = (int64_t)gridDim.x * NG;
  int64_t tok = (int64_t)blockIdx.x * NG + grp;
  auto issue = [&](int64_t tk, int s) {
    const int64_t so = lay.tok_off(tk, D);
    if (lane < T)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(st_s + s * kMaxT + lane)),
                   "l"(p.stats + (int64_t)lane * p.R + tk)
                   : "memory");
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const int64_t rb = ((int64_t)t * p.R + tk) * p.ld;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        cp_async_vec<EBP>(pre_at(s, t, i), reinterpret_cast<const unsigned char*>(p.pre) + (rb + cols[i]) * EBP);
        cp_async_vec<EBG>(gs_at(s, t, i),
                          reinterpret_cast<const unsigned char*>(p.g_spikes) + (so + t * lay.t_stride + coff[i]) * EBG);
      }
    }
  };
#pragma unroll
  for (int k = 0; k < S - 1; ++k) {
    if (tok + k * step < p.R) issue(tok + k * step, k);
    cp_async_commit();
  }
  int s = 0;
  for (; tok < p.R; tok += step, s = s + 1 == S ? 0 : s + 1) {
    const int64_t tn = tok + (S - 1) * step;
    __syncwarp();  // every lane has read the statistics of the stage about to be refilled
    if (tn < p.R) issue(tn, s == 0 ? S - 1 : s - 1);
    cp_async_commit();
    cp_async_wait<S - 1>();  // this token's vectors and statistics have landed
    __syncwarp();            // the statistics were copied by lanes t < T
    float2 nm[kMaxT], rs[kMaxT];
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      const float2 st = t < T ? st_s[s * kMaxT + t] : make_float2(0.0f, 1.0f);
      nm[t] = make_float2(-st.x, -st.x);
      rs[t] = make_float2(st.y, st.y);
    }
    // x^ of every row (kept in shared memory for the two later passes) and
    // the membrane before reset at every step
    float2 u[kMaxT][NV][2];
    {
      float2 v[NV][2];
#pragma unroll
      for (int i = 0; i < NV; ++i) v[i][0] = v[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int t = 0; t < kMaxT; ++t) {
        if (t >= T) continue;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float x[4];
          raw_unpack<EBP>(*pre_at(s, t, i), p.pre_dtype, x);
          float2 xh[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            xh[j] = mul2(add2(add2(make_float2(x[2 * j], x[2 * j + 1]), pb[i][j]), nm[t]), rs[t]);
            const float2 uu = add2(mul2(v[i][j], beta2), fma2(xh[j], gg[i][j], bb[i][j]));
            u[t][i][j] = uu;
            v[i][j] = make_float2(uu.x > vth ? vr : uu.x, uu.y > vth ? vr : uu.y);
          }
          *xh_at(t, i) = make_float4(xh[0].x, xh[0].y, xh[1].x, xh[1].y);
        }
      }
    }
    // BPTT: dL/dv of every row (into u[t], which step t - 1 no longer reads),
    // and each row's sums of g gamma and g gamma x^ (g = gain dL/dv = dL/dy)
    float2 sums[kMaxT];
    {
      float2 gst[NV][2];
#pragma unroll
      for (int i = 0; i < NV; ++i) gst[i][0] = gst[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int t = kMaxT - 1; t >= 0; --t) {
        sums[t] = make_float2(0.0f, 0.0f);
        if (t >= T) continue;
        float2 sa = make_float2(0.0f, 0.0f), sb = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float gsv[4];
          raw_unpack<EBG>(*gs_at(s, t, i), p.gs_dtype, gsv);
          const float4 x4 = *xh_at(t, i);
          const float2 xh[2] = {make_float2(x4.x, x4.y), make_float2(x4.z, x4.w)};
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float2 uu = u[t][i][j];
            const float2 d = add2(uu, nvth2);
            float2 sg;
            if constexpr (SURR == SPK_SURROGATE_SUPERSPIKE) {
              const float2 q = fma2(make_float2(p.k, p.k), make_float2(fabsf(d.x), fabsf(d.y)), make_float2(1.f, 1.f));
              const float2 q2 = mul2(q, q);
              sg = make_float2(__fdividef(1.0f, q2.x), __fdividef(1.0f, q2.y));
            } else {
              const float2 z = mul2(make_float2(p.c_arctan, p.c_arctan), d);
              const float2 den = fma2(z, z, make_float2(1.f, 1.f));
              const float hk = 0.5f * p.k;
              sg = make_float2(__fdividef(hk, den.x), __fdividef(hk, den.y));
            }
            const float2 from = make_float2(uu.x > vth ? 0.0f : gst[i][j].x, uu.y > vth ? 0.0f : gst[i][j].y);
            const float2 gv = fma2(make_float2(gsv[2 * j], gsv[2 * j + 1]), sg, from);
            if (t > 0) {
              const float2 up = u[t - 1][i][j];
              acc_lb = fma2(gv, make_float2(up.x > vth ? vr : up.x, up.y > vth ? vr : up.y), acc_lb);
            }
            gst[i][j] = mul2(gv, beta2);
            u[t][i][j] = gv;
            const float2 gxg = mul2(gv, gg[i][j]);  // dL/dy gamma = dL/dv gain gamma
            sa = add2(sa, gxg);
            sb = fma2(gxg, xh[j], sb);
          }
        }
        sums[t] = make_float2(sa.x + sa.y, sb.x + sb.y);
      }
    }
    warp_sum2(sums, T);
    gx.sum(sums, T, lane);
    // dx = rstd (g gamma - mean(g gamma) - x^ mean(g gamma x^)), and the
    // per-column sums of dL/dv x^, dL/dv and dx
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t >= T) continue;
      const float2 ma = make_float2(-sums[t].x * invD, -sums[t].x * invD);
      const float2 mb = make_float2(-sums[t].y * invD, -sums[t].y * invD);
      const int64_t rb = ((int64_t)t * p.R + tok) * p.ld;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float4 x4 = *xh_at(t, i);
        const float2 xh[2] = {make_float2(x4.x, x4.y), make_float2(x4.z, x4.w)};
        float dx[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 gv = u[t][i][j];
          const float2 dd = mul2(fma2(xh[j], mb, fma2(gv, gg[i][j], ma)), rs[t]);
          dx[2 * j] = dd.x;
          dx[2 * j + 1] = dd.y;
          acc_g[i][j] = fma2(gv, xh[j], acc_g[i][j]);
          acc_b[i][j] = add2(acc_b[i][j], gv);
          acc_d[i][j] = add2(acc_d[i][j], dd);
        }
        store4(p.g_pre, p.pre_dtype, rb + cols[i], dx);
      }
    }
  }
  // block partials: the token groups' column sums added in group order, the
  // LIF beta term over the warps in warp order (the staging memory is reused)
  cp_async_wait<0>();
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [NG][3 D]
  // dL/dgamma = sum dL/dy x^ and dL/dbeta = sum dL/dy, with dL/dy = gain dL/dv
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float* r = red + (size_t)grp * 3 * D + cols[i];
    const float2 g0 = mul2(acc_g[i][0], gain2), g1 = mul2(acc_g[i][1], gain2);
    const float2 b0 = mul2(acc_b[i][0], gain2), b1 = mul2(acc_b[i][1], gain2);
    *reinterpret_cast<float4*>(r) = make_float4(g0.x, g0.y, g1.x, g1.y);
    *reinterpret_cast<float4*>(r + D) = make_float4(b0.x, b0.y, b1.x, b1.y);
    *reinterpret_cast<float4*>(r + 2 * D) = make_float4(acc_d[i][0].x, acc_d[i][0].y, acc_d[i][1].x, acc_d[i][1].y);
  }
  const float lbw = warp_sum(acc_lb.x + acc_lb.y);
  if (lane == 0) lb_red[warp] = lbw;
  __syncthreads();
  float* out = p.part + (int64_t)blockIdx.x * (3 * D + 1);
  for (int c = threadIdx.x; c < 3 * D; c += blockDim.x) {
    float a = red[c];
#pragma unroll
    for (int g = 1; g < NG; ++g) a += red[(size_t)g * 3 * D + c];
    out[c] = a;
  }
  if (threadIdx.x == 0) {
    float a = lb_red[0];
#pragma unroll
    for (int w = 1; w < W; ++w) a += lb_red[w];
    out[3 * D] = a;
  }
}

// column c of the [rows][W] partials (dgamma, dbeta, dbias, LIF beta): 32 row
// groups (rows r = g mod 32, in order) per column, combined in group order
constexpr int kSumGroups = 32;
__global__ void __launch_bounds__(32 * kSumGroups) sum_columns_kernel(const float* __restrict__ part, int rows, int W,
                                                          float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                          float* __restrict__ dbias, float* __restrict__ dlif_beta,
                                                          int D) {
  __shared__ float acc[kSumGroups][33];
  const int cl = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  float s = 0.0f;
  if (c < W)
    for (int r = grp; r < rows; r += kSumGroups) s += part[(int64_t)r * W + c];
  acc[grp][cl] = s;
  __syncthreads();
  if (grp != 0 || c >= W) return;
  s = acc[0][cl];
#pragma unroll
  for (int g = 1; g < kSumGroups; ++g) s += acc[g][cl];
  if (c < D) {
    if (dgamma) dgamma[c] = s;
  } else if (c < 2 * D) {
    if (dbeta) dbeta[c - D] = s;
  } else if (c < 3 * D) {
    if (dbias) dbias[c - 2 * D] = s;
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

// one-token-per-block kernels: D % 128 == 0; persistent grid of up to 64 warps
// (at most 16 blocks) per SM
template <int SURR>
void launch_bwd_tok(bool p32, bool g32, bool pf, int grid, int threads, cudaStream_t st, const BwdParams& p) {
  if (pf) {
    if (p32)
      g32 ? ln_lif_bwd_tok_kernel<4, 4, true, SURR><<<grid, threads, 0, st>>>(p)
          : ln_lif_bwd_tok_kernel<4, 2, true, SURR><<<grid, threads, 0, st>>>(p);
    else
      g32 ? ln_lif_bwd_tok_kernel<2, 4, true, SURR><<<grid, threads, 0, st>>>(p)
          : ln_lif_bwd_tok_kernel<2, 2, true, SURR><<<grid, threads, 0, st>>>(p);
  } else {
    if (p32)
      g32 ? ln_lif_bwd_tok_kernel<4, 4, false, SURR><<<grid, threads, 0, st>>>(p)
          : ln_lif_bwd_tok_kernel<4, 2, false, SURR><<<grid, threads, 0, st>>>(p);
    else
      g32 ? ln_lif_bwd_tok_kernel<2, 4, false, SURR><<<grid, threads, 0, st>>>(p)
          : ln_lif_bwd_tok_kernel<2, 2, false, SURR><<<grid, threads, 0, st>>>(p);
  }
}

inline bool use_tok(int D) { return D % 128 == 0 && D <= 128 * kTokMaxWarps; }
// the one-token-per-block kernels move four elements per vector access and
// read gamma / beta / bias as float4: every pointer 16-byte aligned
inline bool tok_aligned(std::initializer_list<const void*> ptrs) {
  for (const void* q : ptrs)
    if (q && (reinterpret_cast<uintptr_t>(q) & 15) != 0) return false;
  return true;
}
inline int tok_grid(int64_t R, int D) {
  const int nw = D / 128;
  int bps = 64 / nw;
  if (bps > 16) bps = 16;
  const int64_t cap = (int64_t)num_sms() * bps;
  const int64_t g = R < cap ? R : cap;
  return g < 1 ? 1 : (int)g;
}
// token-group kernels: blocks of `warps` warps, warps / G tokens at a time;
// blocks_per_sm resident blocks (the backward holds one per SM)
inline int grp_grid(int64_t R, int D, int blocks_per_sm, int warps = kGrpWarps, int nv = kGrpNV) {
  const int ng = warps / (D / (128 * nv));
  const int64_t need = (R + ng - 1) / ng, cap = (int64_t)num_sms() * blocks_per_sm;
  const int64_t g = need < cap ? need : cap;
  return g < 1 ? 1 : (int)g;
}
constexpr int kGrpFwdBlocksPerSm = 2;
constexpr int kGrpBwdBlocksPerSm = 1;

// token-group backward: warps per block and vectors per lane
inline int bwd_grid(int64_t R, int D, bool aligned16) {
  if (R == 0) return 1;
  if (use_grp(D) && aligned16)
    return grp_grid(R, D, kGrpBwdBlocksPerSm, grp_bwd_warps<kGrpBwdNV>(), kGrpBwdNV);
  return use_tok(D) && aligned16 ? tok_grid(R, D) : grid_blocks(R, pick_nw(D));
}

template <int EB, int SD, int G, bool RESID = false>
int launch_fwd_grp_g(int grid, cudaStream_t st, const FwdParams& p) {
  constexpr size_t smem = (size_t)kGrpWarps * kGrpFwdStages * kMaxT * kGrpNV * 32 * 4 * EB;
  static bool attr_set = false;  // per instantiation; idempotent if two threads race
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(ln_lif_fwd_grp_kernel<EB, SD, G, RESID>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  ln_lif_fwd_grp_kernel<EB, SD, G, RESID><<<grid, 32 * kGrpWarps, smem, st>>>(p);
  return SPK_OK;
}

template <int EB, int SD, bool RESID = false>
int launch_fwd_grp(int D, int grid, cudaStream_t st, const FwdParams& p) {
  if (D == 384) return launch_fwd_grp_g<EB, SD, 1, RESID>(grid, st, p);
  if (D == 768) return launch_fwd_grp_g<EB, SD, 2, RESID>(grid, st, p);
  return launch_fwd_grp_g<EB, SD, 4, RESID>(grid, st, p);
}

template <int EBP, int EBG, int SURR, int NV, int G>
int launch_bwd_grp_g(int grid, cudaStream_t st, const BwdParams& p) {
  constexpr size_t smem = grp_bwd_smem_bytes<EBP, EBG, NV>();
  static_assert(smem >= (size_t)grp_bwd_warps<NV>() * 3 * 128 * NV * sizeof(float),
                "block partials reuse the staging memory");
  static_assert(smem <= 227 * 1024, "staging exceeds the shared memory of a block");
  static bool attr_set = false;  // per instantiation; idempotent if two threads race
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(ln_lif_bwd_grp_kernel<EBP, EBG, SURR, NV, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  ln_lif_bwd_grp_kernel<EBP, EBG, SURR, NV, G><<<grid, 32 * grp_bwd_warps<NV>(), smem, st>>>(p);
  return SPK_OK;
}

template <int EBP, int EBG, int SURR>
int launch_bwd_grp_d(int D, int grid, cudaStream_t st, const BwdParams& p) {
  constexpr int NV = kGrpBwdNV, G1 = 3 / NV;  // warps per token at D = 384
  if (D == 384) return launch_bwd_grp_g<EBP, EBG, SURR, NV, G1>(grid, st, p);
  if (D == 768) return launch_bwd_grp_g<EBP, EBG, SURR, NV, 2 * G1>(grid, st, p);
  return launch_bwd_grp_g<EBP, EBG, SURR, NV, 4 * G1>(grid, st, p);
}

template <int SURR>
int launch_bwd_grp(bool p32, bool g32, int D, int grid, cudaStream_t st, const BwdParams& p) {
  if (p32) return g32 ? launch_bwd_grp_d<4, 4, SURR>(D, grid, st, p) : launch_bwd_grp_d<4, 2, SURR>(D, grid, st, p);
  return g32 ? launch_bwd_grp_d<2, 4, SURR>(D, grid, st, p) : launch_bwd_grp_d<2, 2, SURR>(D, grid, st, p);
}

}  // namespace lnlif

using namespace lnlif;

// pre row stride wider than D (a column slice of a wider GEMM output): only the
// one-token-per-block kernels
static int check_ld(int64_t ld, int64_t D, bool tok_ok) {
  if (ld == D) return SPK_OK;
  SPK_REQUIRE(ld > D && tok_ok, SPK_ERR_SHAPE,
              "pre row stride %lld needs D %% 128 == 0 (D=%lld), a stride >= D and a multiple of 4, and 16-byte "
              "aligned pointers", (long long)ld, (long long)D);
  return SPK_OK;
}

// head-major spike layout (head_dim > 0): only the one-token-per-block kernels
static int check_heads(int64_t head_dim, int64_t seq_len, int64_t R, int D, bool tok_ok) {
  if (head_dim <= 0) return SPK_OK;
  SPK_REQUIRE(tok_ok, SPK_ERR_SHAPE,
              "head-major spikes need D %% 128 == 0 (D=%d) and 16-byte aligned pointers", D);
  SPK_REQUIRE(head_dim % 4 == 0 && D % head_dim == 0 && seq_len >= 1 && R % seq_len == 0 && R < (1ll << 31),
              SPK_ERR_SHAPE,
              "head-major spikes: head_dim=%lld must be a multiple of 4 dividing D=%d, and seq_len=%lld must "
              "divide R=%lld", (long long)head_dim, D, (long long)seq_len, (long long)R);
  return SPK_OK;
}

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
  if (D < 32 || D > 4 * 32 * spk::lnlif::kMaxCpt || R < 0) return 0;
  // the largest of the backward's possible grids on the current device (one
  // partial row per block); fewer warps per block give more blocks
  const int g1 = spk::lnlif::bwd_grid(R, (int)D, true), g2 = spk::lnlif::bwd_grid(R, (int)D, false);
  return (int64_t)(g1 > g2 ? g1 : g2) * (3 * D + 1) * (int64_t)sizeof(float);
}

int spk_ln_lif_fwd(const void* pre, int pre_dtype, const float* pre_bias, const float* ln_gamma,
                   const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                   const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t D, int64_t pre_ld,
                   int64_t head_dim, int64_t seq_len, void* spikes, int spike_dtype, float* stats, void* stream) {
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
  FwdParams p = {pre, pre_dtype, pre_bias, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vreset, in_gain,
                 spikes, spike_dtype, reinterpret_cast<float2*>(stats), (int)T, R, (int)D, 0,
                 (int)(head_dim > 0 ? head_dim : 0), (int)(seq_len > 0 ? seq_len : 1), pre_ld > 0 ? pre_ld : D};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool aligned16 = tok_aligned({pre, spikes, ln_gamma, ln_beta, pre_bias}) && p.ld % 4 == 0;
  if ((rc = check_ld(p.ld, D, use_tok((int)D) && aligned16)) != SPK_OK) return rc;
  SPK_REQUIRE(aligned16 || D <= 32 * kMaxCpt, SPK_ERR_ALIGN,
              "D=%lld > %d needs pre, spikes, ln_gamma, ln_beta and pre_bias 16-byte aligned", (long long)D,
              32 * kMaxCpt);
  if ((rc = check_heads(head_dim, seq_len, R, (int)D, use_tok((int)D) && aligned16)) != SPK_OK) return rc;
  if (use_grp((int)D) && aligned16) {
    const int grid = grp_grid(R, (int)D, pre_dtype == SPK_F32 ? 1 : kGrpFwdBlocksPerSm);
    if (pre_dtype == SPK_F32) {
      rc = spike_dtype == SPK_F32    ? launch_fwd_grp<4, SPK_F32>((int)D, grid, st, p)
           : spike_dtype == SPK_BF16 ? launch_fwd_grp<4, SPK_BF16>((int)D, grid, st, p)
                                     : launch_fwd_grp<4, -1>((int)D, grid, st, p);
    } else {
      rc = spike_dtype == SPK_F32    ? launch_fwd_grp<2, SPK_F32>((int)D, grid, st, p)
           : spike_dtype == SPK_BF16 ? launch_fwd_grp<2, SPK_BF16>((int)D, grid, st, p)
                                     : launch_fwd_grp<2, -1>((int)D, grid, st, p);
    }
    if (rc != SPK_OK) return rc;
  } else if (use_tok((int)D) && aligned16) {
    const int grid = tok_grid(R, (int)D), threads = (int)D / 4;
    if (pre_dtype == SPK_F32) {
      spike_dtype == SPK_F32 ? ln_lif_fwd_tok_kernel<4, SPK_F32><<<grid, threads, 0, st>>>(p)
      : spike_dtype == SPK_BF16 ? ln_lif_fwd_tok_kernel<4, SPK_BF16><<<grid, threads, 0, st>>>(p)
                                : ln_lif_fwd_tok_kernel<4, -1><<<grid, threads, 0, st>>>(p);
    } else {
      spike_dtype == SPK_F32 ? ln_lif_fwd_tok_kernel<2, SPK_F32><<<grid, threads, 0, st>>>(p)
      : spike_dtype == SPK_BF16 ? ln_lif_fwd_tok_kernel<2, SPK_BF16><<<grid, threads, 0, st>>>(p)
                                : ln_lif_fwd_tok_kernel<2, -1><<<grid, threads, 0, st>>>(p);
    }
  } else {
    // D not a multiple of 128 (so D <= 512): one warp per token, single columns
    const int nw = pick_nw((int)D);
    p.cpt = (int)D / (32 * nw);
    ln_lif_fwd_kernel<1, 1, kMaxCpt><<<grid_blocks(R, nw, 8), kThreads, 0, st>>>(p);
  }
  return check_launch("ln_lif_fwd_kernel");
}

int spk_ln_lif_fwd_residual(const void* pre, int pre_dtype, const float* pre_bias, const float* ln_gamma,
                            const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                            const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t D, int64_t pre_ld,
                            const float* residual, float* out, void* out_bf16, float* stats, void* stream) {
  using namespace spk;
  int rc = check_ln_lif((int)T, R, (int)D);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE((pre && residual && out && stats) || R == 0, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(lif_beta && lif_vth && lif_vreset, SPK_ERR_INVALID, "null LIF parameter");
  SPK_REQUIRE(pre_dtype == SPK_F32 || pre_dtype == SPK_F16 || pre_dtype == SPK_BF16, SPK_ERR_INVALID,
              "pre dtype %d not supported", pre_dtype);
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  if (R == 0) return SPK_OK;
  const int64_t ld = pre_ld > 0 ? pre_ld : D;
  const bool aligned16 = tok_aligned({pre, residual, out, out_bf16, ln_gamma, ln_beta, pre_bias}) && ld % 4 == 0;
  if (!(use_grp((int)D) && aligned16))
    return fail(SPK_ERR_UNSUPPORTED, "residual form needs D in {384, 768, 1536} and 16-byte aligned pointers");
  FwdParams p = {pre, pre_dtype, pre_bias, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vreset, in_gain,
                 out, SPK_F32, reinterpret_cast<float2*>(stats), (int)T, R, (int)D, 0, 0, 1, ld,
                 residual, reinterpret_cast<__nv_bfloat16*>(out_bf16)};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grid = grp_grid(R, (int)D, pre_dtype == SPK_F32 ? 1 : kGrpFwdBlocksPerSm);
  rc = pre_dtype == SPK_F32 ? launch_fwd_grp<4, SPK_F32, true>((int)D, grid, st, p)
                            : launch_fwd_grp<2, SPK_F32, true>((int)D, grid, st, p);
  if (rc != SPK_OK) return rc;
  return check_launch("ln_lif_fwd_grp_kernel");
}

int spk_ln_lif_bwd(const void* g_spikes, int gs_dtype, const void* pre, int pre_dtype, const float* pre_bias,
                   const float* stats, const float* ln_gamma, const float* ln_beta, const float* lif_beta,
                   const float* lif_vth, const float* lif_vreset, float in_gain, int surrogate, float surrogate_k,
                   int64_t T, int64_t R, int64_t D, int64_t pre_ld, int64_t head_dim, int64_t seq_len, void* g_pre,
                   float* g_gamma,
                   float* g_beta_ln, float* g_bias, float* g_lif_beta, void* workspace, int64_t workspace_bytes,
                   void* stream) {
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
  const int64_t ld = pre_ld > 0 ? pre_ld : D;
  const bool aligned16 = tok_aligned({g_spikes, pre, g_pre, ln_gamma, ln_beta, pre_bias}) && ld % 4 == 0;
  if ((rc = check_ld(ld, D, use_tok((int)D) && aligned16)) != SPK_OK) return rc;
  SPK_REQUIRE(aligned16 || D <= 32 * kMaxCpt, SPK_ERR_ALIGN,
              "D=%lld > %d needs g_spikes, pre, g_pre, ln_gamma, ln_beta and pre_bias 16-byte aligned",
              (long long)D, 32 * kMaxCpt);
  if ((rc = check_heads(head_dim, seq_len, R, (int)D, use_tok((int)D) && aligned16)) != SPK_OK) return rc;
  const int grid = bwd_grid(R, (int)D, aligned16);
  SPK_REQUIRE((int64_t)grid * (3 * D + 1) * 4 <= workspace_bytes, SPK_ERR_INVALID, "workspace too small for %d blocks",
              grid);
  float* part = reinterpret_cast<float*>(workspace);
  if (R == 0) {
    cudaError_t e = cudaMemsetAsync(part, 0, (size_t)(3 * D + 1) * 4, st);
    if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  } else {
    BwdParams p = {g_spikes, gs_dtype, pre, pre_dtype, pre_bias, reinterpret_cast<const float2*>(stats), ln_gamma,
                   ln_beta, lif_beta, lif_vth, lif_vreset, in_gain, surrogate, surrogate_k,
                   (float)(3.14159265358979323846 / 2.0 * (double)surrogate_k), g_pre, part, (int)T, R, (int)D, 0,
                   (int)(head_dim > 0 ? head_dim : 0), (int)(seq_len > 0 ? seq_len : 1), pre_ld > 0 ? pre_ld : D};
    if (use_grp((int)D) && aligned16) {
      const bool p32 = pre_dtype == SPK_F32, g32 = gs_dtype == SPK_F32;
      rc = surrogate == SPK_SURROGATE_ARCTAN ? launch_bwd_grp<SPK_SURROGATE_ARCTAN>(p32, g32, (int)D, grid, st, p)
                                             : launch_bwd_grp<SPK_SURROGATE_SUPERSPIKE>(p32, g32, (int)D, grid, st, p);
      if (rc != SPK_OK) return rc;
    } else if (use_tok((int)D) && aligned16) {
      const int threads = (int)D / 4;
      const bool p32 = pre_dtype == SPK_F32, g32 = gs_dtype == SPK_F32;
      if (surrogate == SPK_SURROGATE_ARCTAN)
        launch_bwd_tok<SPK_SURROGATE_ARCTAN>(p32, g32, D <= 128 * kTokPfWarps, grid, threads, st, p);
      else
        launch_bwd_tok<SPK_SURROGATE_SUPERSPIKE>(p32, g32, D <= 128 * kTokPfWarps, grid, threads, st, p);
    } else {
      // D not a multiple of 128 (so D <= 512): one warp per token, single columns
      p.cpt = (int)D / 32;
      ln_lif_bwd_kernel<1, 1, kMaxCpt><<<grid, kThreads, 0, st>>>(p);
    }
    if ((rc = check_launch("ln_lif_bwd_kernel")) != SPK_OK) return rc;
  }
  const int W = 3 * (int)D + 1;
  sum_columns_kernel<<<(W + 31) / 32, 32 * kSumGroups, 0, st>>>(part, grid, W, g_gamma, g_beta_ln, g_bias,
                                                                  g_lif_beta, (int)D);
  return check_launch("sum_columns_kernel");
}

}  // extern "C"
