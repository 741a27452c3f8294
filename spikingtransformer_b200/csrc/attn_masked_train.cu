// Masked spiking attention for training, short sequences (Nq, Nk <= 64):
// forward and backward of the attention core in one CTA per (t*b, head).
//
// Reference: Triton_Layers/SSA.py:234-242 (XNOR scores :145-165, log-distance
// bias :177-201, "+ bias, * mask, * scale, @ V") and the plain form
// SSA.py:81-84, differentiated by torch's autograd in the reference
// (train_spikeformer.py:561).  The decoder's masked self-attention
// (Decoder.py:18) is the caller: Nq = Nk = 64 in the OCR model.
//
//   S_ij = dh - |q_i| - |k_j| + 2 q_i.k_j + R(|i-j|)   (XNOR; plain: q_i.k_j)
//   P = S * M (mask 0/1),  a = scale * P V
// Backward, with G = dL/da:
//   D = G V^T,  dscale = sum(P * D),  dS = scale * D * M,
//   dV = scale * P^T G,
//   dQ = dS (2K - 1) and dK = dS^T (2Q - 1)   (XNOR; plain: dS K, dS^T Q).
// Spikes are 0/1, so S, P and P V are exact integers in fp32; everything else
// is fp32 arithmetic on the CUDA cores (the score matrix never leaves shared
// memory).
#include "common.cuh"

namespace spk {
namespace amt {

constexpr int kThreads = 256;
constexpr int kMaxN = 64;
constexpr int kMaxD = 64;
constexpr int kS = 68;  // row stride (floats) of every [64][64] tile: 16-byte rows, 4-way LDS.128 at most

template <typename X> struct ElemCode;
template <> struct ElemCode<float> { static constexpr int code = SPK_F32; };
template <> struct ElemCode<__half> { static constexpr int code = SPK_F16; };
template <> struct ElemCode<__nv_bfloat16> { static constexpr int code = SPK_BF16; };

struct Params {
  int TB, B, H, Nq, Nk, dh, variant, lmax;
  int64_t q_st, q_sh, q_sn;  // element strides of q (t*b, head, position); d stride 1
  int64_t k_st, k_sh, k_sn;
  int64_t v_st, v_sh, v_sn;
  const uint8_t* mask;       // nullptr: no mask; else element (t,b,h,i,j) at t*m_st+b*m_sb+h*m_sh+i*m_sq+j
  int64_t m_st, m_sb, m_sh, m_sq;
  const float* scale;
  int vec;                   // q, k, v rows may be read and written 4 elements at a time
};

constexpr int kTile = kMaxN * kS;  // floats per tile

// shared memory: the forward uses q, k, v, P; the backward also G, P^T and dS^T
__host__ __device__ inline size_t smem_bytes(bool bwd) {
  return (size_t)(bwd ? 7 : 4) * kTile * sizeof(float) + 2 * kMaxN * sizeof(float) + kMaxN;
}

// 4 consecutive elements of a row as float4 (vector path: 4-element aligned)
template <typename X>
__device__ inline float4 load4(const X* p, bool vec, int n_valid) {
  if (vec && n_valid >= 4) {
    if constexpr (sizeof(X) == 4) {
      return *reinterpret_cast<const float4*>(p);
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      const X* e = reinterpret_cast<const X*>(&w);
      return make_float4(Elem<ElemCode<X>::code>::load(e), Elem<ElemCode<X>::code>::load(e + 1),
                         Elem<ElemCode<X>::code>::load(e + 2), Elem<ElemCode<X>::code>::load(e + 3));
    }
  }
  float f[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) f[u] = u < n_valid ? Elem<ElemCode<X>::code>::load(p + u) : 0.0f;
  return make_float4(f[0], f[1], f[2], f[3]);
}

template <typename X>
__device__ inline void store4(X* p, float4 v, bool vec, int n_valid) {
  if (vec && n_valid >= 4) {
    if constexpr (sizeof(X) == 4) {
      *reinterpret_cast<float4*>(p) = v;
    } else {
      X e[4] = {Elem<ElemCode<X>::code>::make(v.x), Elem<ElemCode<X>::code>::make(v.y),
                Elem<ElemCode<X>::code>::make(v.z), Elem<ElemCode<X>::code>::make(v.w)};
      *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(e);
    }
    return;
  }
  const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (u < n_valid) p[u] = Elem<ElemCode<X>::code>::make(f[u]);
}

// rows [0, n) of a [n][dh] operand (row stride sn) into a zero-padded [64][kS] tile
template <typename X>
__device__ inline void load_tile(const X* src, int64_t sn, int n, int dh, bool vec, float* dst) {
  for (int e = threadIdx.x; e < kMaxN * (kMaxD / 4); e += kThreads) {
    const int r = e >> 4, c = (e & 15) * 4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (r < n && c < dh) v = load4(src + r * sn + c, vec, dh - c);
    *reinterpret_cast<float4*>(dst + r * kS + c) = v;
  }
}

// C[i][c0 + u] = sum_d A[i][d] B[c0 + u][d], u < 16, d < dlen (a multiple of 4):
// thread row i = tid % 64, column group c0 = 16 (tid / 64), the same in a warp
// (B rows broadcast); A rows are 16-byte loads.
__device__ inline void gemm_rt(const float* A, const float* B, int dlen, float (&acc)[16]) {
  const int i = threadIdx.x & 63, c0 = (threadIdx.x >> 6) * 16;
#pragma unroll
  for (int u = 0; u < 16; ++u) acc[u] = 0.0f;
  for (int d = 0; d < dlen; d += 4) {
    const float4 a = *reinterpret_cast<const float4*>(A + i * kS + d);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float4 b = *reinterpret_cast<const float4*>(B + (c0 + u) * kS + d);
      acc[u] = fmaf(a.x, b.x, acc[u]);
      acc[u] = fmaf(a.y, b.y, acc[u]);
      acc[u] = fmaf(a.z, b.z, acc[u]);
      acc[u] = fmaf(a.w, b.w, acc[u]);
    }
  }
}

// C[i][c0 + u] = sum_j A[i][j] B[j][c0 + u], j < jlen (a multiple of 4); also
// returns sum_j A[i][j]
__device__ inline float gemm_rn(const float* A, const float* B, int jlen, float (&acc)[16]) {
  const int i = threadIdx.x & 63, c0 = (threadIdx.x >> 6) * 16;
  float asum = 0.0f;
#pragma unroll
  for (int u = 0; u < 16; ++u) acc[u] = 0.0f;
  for (int j = 0; j < jlen; j += 4) {
    const float4 a = *reinterpret_cast<const float4*>(A + i * kS + j);
    asum += (a.x + a.y) + (a.z + a.w);
    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const float4* brow = reinterpret_cast<const float4*>(B + (j + jj) * kS + c0);
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        const float4 b = brow[u4];
        acc[4 * u4 + 0] = fmaf(av[jj], b.x, acc[4 * u4 + 0]);
        acc[4 * u4 + 1] = fmaf(av[jj], b.y, acc[4 * u4 + 1]);
        acc[4 * u4 + 2] = fmaf(av[jj], b.z, acc[4 * u4 + 2]);
        acc[4 * u4 + 3] = fmaf(av[jj], b.w, acc[4 * u4 + 3]);
      }
    }
  }
  return asum;
}

__device__ inline int round4(int n) { return (n + 3) & ~3; }

struct Unit {
  float *q, *k, *v, *p;
  float *rq, *rk;
  unsigned char* rl;
};

// q, k, v of a unit into shared memory, their row sums, then P = S * M
// (written at P[i][j], and at Pt[j][i] when Pt is given)
template <typename X>
__device__ inline void scores(const Params& p, const X* q, const X* k, const X* v, int unit, const Unit& u,
                              float* pt) {
  const int tb = unit / p.H, h = unit % p.H;
  const bool vec = p.vec != 0;
  load_tile(q + tb * p.q_st + h * p.q_sh, p.q_sn, p.Nq, p.dh, vec, u.q);
  load_tile(k + tb * p.k_st + h * p.k_sh, p.k_sn, p.Nk, p.dh, vec, u.k);
  load_tile(v + tb * p.v_st + h * p.v_sh, p.v_sn, p.Nk, p.dh, vec, u.v);
  __syncthreads();
  if (threadIdx.x < 2 * kMaxN) {
    const int r = threadIdx.x & (kMaxN - 1);
    const float* row = (threadIdx.x < kMaxN ? u.q : u.k) + r * kS;
    float s = 0.0f;
    for (int d = 0; d < p.dh; ++d) s += row[d];
    (threadIdx.x < kMaxN ? u.rq : u.rk)[r] = s;
  }
  __syncthreads();
  float acc[16];
  gemm_rt(u.q, u.k, round4(p.dh), acc);
  const int i = threadIdx.x & 63, c0 = (threadIdx.x >> 6) * 16;
  const int t_idx = tb / p.B, b = tb % p.B;
  const uint8_t* mrow = p.mask ? p.mask + t_idx * p.m_st + b * p.m_sb + h * p.m_sh + (int64_t)i * p.m_sq : nullptr;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const int j = c0 + w;
    float s = acc[w];
    if (p.variant == 1) {
      const int dist = i > j ? i - j : j - i;
      s = ((float)p.dh - (u.rq[i] + u.rk[j] - 2.0f * s)) + (dist < p.lmax ? (float)u.rl[dist] : 0.0f);
    }
    bool keep = i < p.Nq && j < p.Nk;
    if (keep && mrow) keep = mrow[j] != 0;
    const float pv = keep ? s : 0.0f;
    u.p[i * kS + j] = pv;
    if (pt) pt[j * kS + i] = pv;
  }
  __syncthreads();
}

__device__ inline void log_distance_table(int lmax, unsigned char* rl) {
  if (threadIdx.x < kMaxN) {
    // R(d) = the smallest r >= 0 with (d + 1) * 2^r >= L - 1
    int r = 0, x = threadIdx.x + 1;
    while (x < lmax - 1) {
      x <<= 1;
      ++r;
    }
    rl[threadIdx.x] = (unsigned char)r;
  }
}

template <typename X>
__global__ void __launch_bounds__(kThreads) masked_attn_fwd_kernel(const X* __restrict__ q, const X* __restrict__ k,
                                                                   const X* __restrict__ v, float* __restrict__ a,
                                                                   Params p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* f = reinterpret_cast<float*>(smem);
  Unit u;
  u.q = f;
  u.k = f + kTile;
  u.v = f + 2 * kTile;
  u.p = f + 3 * kTile;
  u.rq = f + 4 * kTile;
  u.rk = u.rq + kMaxN;
  u.rl = reinterpret_cast<unsigned char*>(u.rk + kMaxN);
  log_distance_table(p.lmax, u.rl);
  const float scale = __ldg(p.scale);
  const int D = p.H * p.dh;
  const int i = threadIdx.x & 63, c0 = (threadIdx.x >> 6) * 16;
  for (int unit = blockIdx.x; unit < p.TB * p.H; unit += gridDim.x) {
    scores(p, q, k, v, unit, u, nullptr);
    const int tb = unit / p.H, h = unit % p.H;
    float acc[16];
    gemm_rn(u.p, u.v, round4(p.Nk), acc);  // P V (exact integers)
    if (i < p.Nq) {
      float* dst = a + ((int64_t)tb * p.Nq + i) * D + (int64_t)h * p.dh;
#pragma unroll
      for (int w = 0; w < 16; w += 4)
        if (c0 + w < p.dh)
          store4(dst + c0 + w, make_float4(acc[w] * scale, acc[w + 1] * scale, acc[w + 2] * scale, acc[w + 3] * scale),
                 true, p.dh - (c0 + w));
    }
    __syncthreads();
  }
}

template <typename X>
__global__ void __launch_bounds__(kThreads) masked_attn_bwd_kernel(
    const X* __restrict__ q, const X* __restrict__ k, const X* __restrict__ v, const float* __restrict__ g,
    X* __restrict__ dq, X* __restrict__ dk, X* __restrict__ dv, float* __restrict__ dscale_part, Params p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* f = reinterpret_cast<float*>(smem);
  Unit u;
  u.q = f;
  u.k = f + kTile;
  u.v = f + 2 * kTile;
  u.p = f + 3 * kTile;   // P, then dS
  float* gt = f + 4 * kTile;
  float* pt = f + 5 * kTile;
  float* st = f + 6 * kTile;  // dS^T
  u.rq = f + 7 * kTile;
  u.rk = u.rq + kMaxN;
  u.rl = reinterpret_cast<unsigned char*>(u.rk + kMaxN);
  __shared__ float red[kThreads / 32];
  log_distance_table(p.lmax, u.rl);
  const float scale = __ldg(p.scale);
  const int D = p.H * p.dh;
  const int i = threadIdx.x & 63, c0 = (threadIdx.x >> 6) * 16;
  const bool vec = p.vec != 0;
  for (int unit = blockIdx.x; unit < p.TB * p.H; unit += gridDim.x) {
    const int tb = unit / p.H, h = unit % p.H;
    // G of the unit: token-major rows of a, fp32
    for (int e = threadIdx.x; e < kMaxN * (kMaxD / 4); e += kThreads) {
      const int r = e >> 4, c = (e & 15) * 4;
      float4 w = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (r < p.Nq && c < p.dh) w = load4(g + ((int64_t)tb * p.Nq + r) * D + (int64_t)h * p.dh + c, true, p.dh - c);
      *reinterpret_cast<float4*>(gt + r * kS + c) = w;
    }
    scores(p, q, k, v, unit, u, pt);  // synchronises after the G tile too
    // D = G V^T; dscale = sum P * D; dS = scale * D where the mask keeps (P's zeros mark
    // the masked and out-of-range entries only where S happens to be 0 too, so the mask is
    // read again)
    float acc[16];
    gemm_rt(gt, u.v, round4(p.dh), acc);
    const int t_idx = tb / p.B, b = tb % p.B;
    const uint8_t* mrow = p.mask ? p.mask + t_idx * p.m_st + b * p.m_sb + h * p.m_sh + (int64_t)i * p.m_sq : nullptr;
    float ds_sum = 0.0f;
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      const int j = c0 + w;
      bool keep = i < p.Nq && j < p.Nk;
      if (keep && mrow) keep = mrow[j] != 0;
      ds_sum = fmaf(u.p[i * kS + j], acc[w], ds_sum);
      const float dsv = keep ? acc[w] * scale : 0.0f;
      u.p[i * kS + j] = dsv;
      st[j * kS + i] = dsv;
    }
    // per-unit dscale partial, reduced in a fixed order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ds_sum += __shfl_xor_sync(0xffffffffu, ds_sum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ds_sum;
    __syncthreads();
    if (threadIdx.x == 0) {
      float r = 0.0f;
      for (int w = 0; w < kThreads / 32; ++w) r += red[w];
      dscale_part[unit] = r;
    }
    // dV = scale P^T G (thread row = key j)
    gemm_rn(pt, gt, round4(p.Nq), acc);
    if (i < p.Nk) {
      X* dst = dv + tb * p.v_st + h * p.v_sh + i * p.v_sn;
#pragma unroll
      for (int w = 0; w < 16; w += 4)
        if (c0 + w < p.dh)
          store4(dst + c0 + w, make_float4(acc[w] * scale, acc[w + 1] * scale, acc[w + 2] * scale, acc[w + 3] * scale),
                 vec, p.dh - (c0 + w));
    }
    // dQ = dS (2K - 1) (plain: dS K), thread row = query i
    {
      const float rs = gemm_rn(u.p, u.k, round4(p.Nk), acc);
      if (i < p.Nq) {
        X* dst = dq + tb * p.q_st + h * p.q_sh + i * p.q_sn;
#pragma unroll
        for (int w = 0; w < 16; w += 4) {
          float4 o = make_float4(acc[w], acc[w + 1], acc[w + 2], acc[w + 3]);
          if (p.variant == 1) o = make_float4(2.0f * o.x - rs, 2.0f * o.y - rs, 2.0f * o.z - rs, 2.0f * o.w - rs);
          if (c0 + w < p.dh) store4(dst + c0 + w, o, vec, p.dh - (c0 + w));
        }
      }
    }
    // dK = dS^T (2Q - 1) (plain: dS^T Q), thread row = key j
    {
      const float cs = gemm_rn(st, u.q, round4(p.Nq), acc);
      if (i < p.Nk) {
        X* dst = dk + tb * p.k_st + h * p.k_sh + i * p.k_sn;
#pragma unroll
        for (int w = 0; w < 16; w += 4) {
          float4 o = make_float4(acc[w], acc[w + 1], acc[w + 2], acc[w + 3]);
          if (p.variant == 1) o = make_float4(2.0f * o.x - cs, 2.0f * o.y - cs, 2.0f * o.z - cs, 2.0f * o.w - cs);
          if (c0 + w < p.dh) store4(dst + c0 + w, o, vec, p.dh - (c0 + w));
        }
      }
    }
    __syncthreads();
  }
}

template <typename X>
int launch(bool bwd, const void* q, const void* k, const void* v, const Params& p, const float* g, void* dq, void* dk,
           void* dv, float* dscale_part, float* a, cudaStream_t st) {
  const size_t smem = smem_bytes(bwd);
  const int units = p.TB * p.H;
  int grid = num_sms() * 3;
  if (grid > units) grid = units;
  cudaError_t e;
  if (bwd) {
    e = cudaFuncSetAttribute(masked_attn_bwd_kernel<X>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    masked_attn_bwd_kernel<X><<<grid, kThreads, smem, st>>>(
        reinterpret_cast<const X*>(q), reinterpret_cast<const X*>(k), reinterpret_cast<const X*>(v), g,
        reinterpret_cast<X*>(dq), reinterpret_cast<X*>(dk), reinterpret_cast<X*>(dv), dscale_part, p);
    return check_launch("masked_attn_bwd_kernel");
  }
  e = cudaFuncSetAttribute(masked_attn_fwd_kernel<X>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  masked_attn_fwd_kernel<X><<<grid, kThreads, smem, st>>>(reinterpret_cast<const X*>(q), reinterpret_cast<const X*>(k),
                                                          reinterpret_cast<const X*>(v), a, p);
  return check_launch("masked_attn_fwd_kernel");
}

int run(bool bwd, const void* q, const void* k, const void* v, int dtype, const int64_t* strides,
        const uint8_t* mask, int64_t m_st, int64_t m_sb, int64_t m_sh, int64_t m_sq, int variant, const float* scale,
        int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, const float* g, void* dq, void* dk,
        void* dv, float* dscale_part, float* a, void* stream) {
  SPK_REQUIRE(q && k && v && strides && scale, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(bwd ? (g && dq && dk && dv && dscale_part) : (a != nullptr), SPK_ERR_INVALID, "null output");
  SPK_REQUIRE(variant == 0 || variant == 1, SPK_ERR_INVALID, "variant must be 0 (plain) or 1 (xnor)");
  SPK_REQUIRE(dtype == SPK_F32 || dtype == SPK_F16 || dtype == SPK_BF16, SPK_ERR_INVALID, "dtype %d", dtype);
  SPK_REQUIRE(T >= 1 && B >= 1 && H >= 1 && Nq >= 1 && Nk >= 1 && Nq <= kMaxN && Nk <= kMaxN && dh >= 4 &&
                  dh <= kMaxD && dh % 4 == 0 && T * B * H < (1ll << 31),
              SPK_ERR_SHAPE, "unsupported sizes (Nq, Nk <= %d, dh <= %d and a multiple of 4)", kMaxN, kMaxD);
  SPK_REQUIRE(!bwd || aligned(g, 16), SPK_ERR_ALIGN, "g must be 16-byte aligned");
  SPK_REQUIRE(bwd || aligned(a, 16), SPK_ERR_ALIGN, "a must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Params p = {};
  p.TB = (int)(T * B);
  p.B = (int)B;
  p.H = (int)H;
  p.Nq = (int)Nq;
  p.Nk = (int)Nk;
  p.dh = (int)dh;
  p.variant = variant;
  p.lmax = (int)(Nq > Nk ? Nq : Nk);
  p.q_st = strides[0];
  p.q_sh = strides[1];
  p.q_sn = strides[2];
  p.k_st = strides[3];
  p.k_sh = strides[4];
  p.k_sn = strides[5];
  p.v_st = strides[6];
  p.v_sh = strides[7];
  p.v_sn = strides[8];
  p.mask = mask;
  p.m_st = m_st;
  p.m_sb = m_sb;
  p.m_sh = m_sh;
  p.m_sq = m_sq;
  p.scale = scale;
  // 4-element row accesses: 4-aligned strides and pointers (the element size times 4)
  const int es = dtype == SPK_F32 ? 4 : 2;
  bool vec = aligned(q, 4 * es) && aligned(k, 4 * es) && aligned(v, 4 * es);
  if (bwd) vec = vec && aligned(dq, 4 * es) && aligned(dk, 4 * es) && aligned(dv, 4 * es);
  for (int i = 0; i < 9; ++i) vec = vec && strides[i] % 4 == 0;
  p.vec = vec ? 1 : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SPK_F32: return launch<float>(bwd, q, k, v, p, g, dq, dk, dv, dscale_part, a, st);
    case SPK_F16: return launch<__half>(bwd, q, k, v, p, g, dq, dk, dv, dscale_part, a, st);
    default: return launch<__nv_bfloat16>(bwd, q, k, v, p, g, dq, dk, dv, dscale_part, a, st);
  }
}

}  // namespace amt
}  // namespace spk

extern "C" {

int spk_attn_masked_train_fwd(const void* q, const void* k, const void* v, int dtype, const int64_t* strides,
                              const uint8_t* mask, int64_t mask_stride_t, int64_t mask_stride_b,
                              int64_t mask_stride_h, int64_t mask_stride_q, int variant, const float* scale,
                              int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, float* a,
                              void* stream) {
  return spk::amt::run(false, q, k, v, dtype, strides, mask, mask_stride_t, mask_stride_b, mask_stride_h,
                       mask_stride_q, variant, scale, T, B, H, Nq, Nk, dh, nullptr, nullptr, nullptr, nullptr,
                       nullptr, a, stream);
}

int spk_attn_masked_train_bwd(const void* q, const void* k, const void* v, int dtype, const int64_t* strides,
                              const uint8_t* mask, int64_t mask_stride_t, int64_t mask_stride_b,
                              int64_t mask_stride_h, int64_t mask_stride_q, int variant, const float* scale,
                              int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, const float* g,
                              void* dq, void* dk, void* dv, float* dscale_part, void* stream) {
  return spk::amt::run(true, q, k, v, dtype, strides, mask, mask_stride_t, mask_stride_b, mask_stride_h,
                       mask_stride_q, variant, scale, T, B, H, Nq, Nk, dh, g, dq, dk, dv, dscale_part, nullptr,
                       stream);
}

}  // extern "C"
