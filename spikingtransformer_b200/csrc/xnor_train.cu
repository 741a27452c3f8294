// Memory-bound pieces of the training-path XNOR attention core (the
// score-free regrouping of SSA.py:145-165, :177-201, :235-240 used for
// autograd).  The products themselves run as library GEMMs on bf16 operands
// with fp32 accumulation; these kernels fuse everything between them into
// three passes:
//
//   combine:      out[tb, n, h, :] = (QM[b, n, :] + RV[n, b, :] + w[b, :]) * scale
//                 (b = tb*H + h), written token-major [TB][Nq][H][dh], the layout
//                 the output projection reads.  QM, RV and w are exact integers
//                 in fp32, so the sum is exact and the one multiply rounds once.
//   grad_prep:    gs = g * scale from the token-major gradient g, split into
//                 bf16 hi + lo (hi = bf16(gs), lo = bf16(gs - hi)), written
//                 head-major [B][Nq][2 dh] (hi | lo) and n-major
//                 [Nq][2][B][dh] (the operand of the shared log-distance
//                 product); per-chunk column sums of gs and per-thread partial
//                 sums of g * out (for the scale gradient).
//   grad_finish:  dv = KE + RG (n-major) + u, and dk cast to the spike dtype.
//
// The *_lif variants also run the attention's output LIF (lifs, SSA.py:242;
// v_th 0.5): combine_lif scans the T steps of each neuron in registers and
// writes its spikes (for the output projection) besides the pre-activation;
// grad_prep_lif recomputes the membrane from the pre-activation and runs the
// BPTT (the LIF backward of Lif.py:46-102) before the split.  Both keep the
// LIF kernels' operation order (separately rounded multiply and add, IEEE
// division in the surrogate), so they equal the unfused composition bit for
// bit.
#include <type_traits>

#include "common.cuh"

namespace spk {
namespace xnort {

constexpr int kChunk = 16;  // rows of n per grad_prep thread (column-sum partials)

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ qm, const float* __restrict__ rv,
                                                      const float* __restrict__ w, const float* __restrict__ scale,
                                                      float* __restrict__ out, int64_t TB, int H, int Nq, int dh) {
  const int dq4 = dh / 4;
  const int64_t B = TB * H;
  const int64_t total = TB * Nq * H * dq4;
  const float s = __ldg(scale);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    // token-major order: i = ((tb * Nq + n) * H + h) * dq4 + d4
    const int d4 = (int)(i % dq4);
    int64_t r = i / dq4;
    const int h = (int)(r % H);
    r /= H;
    const int n = (int)(r % Nq);
    const int64_t tb = r / Nq;
    const int64_t b = tb * H + h;
    const float4 a = ld4(qm + (b * Nq + n) * dh + 4 * d4);
    const float4 c = ld4(rv + ((int64_t)n * B + b) * dh + 4 * d4);
    const float4 e = ld4(w + b * dh + 4 * d4);
    float4 o;
    o.x = ((a.x + c.x) + e.x) * s;
    o.y = ((a.y + c.y) + e.y) * s;
    o.z = ((a.z + c.z) + e.z) * s;
    o.w = ((a.w + c.w) + e.w) * s;
    *reinterpret_cast<float4*>(out + i * 4) = o;
  }
}

__device__ __forceinline__ void split4(float4 v, uint2& hi, uint2& lo) {
  const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
  const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
  hi.x = *reinterpret_cast<const uint32_t*>(&h0);
  hi.y = *reinterpret_cast<const uint32_t*>(&h1);
  lo.x = *reinterpret_cast<const uint32_t*>(&l0);
  lo.y = *reinterpret_cast<const uint32_t*>(&l1);
}

// grid: x over (tb, h, d4) = B * dh/4 threads, y over chunks of kChunk rows
__global__ void __launch_bounds__(256) grad_prep_kernel(const float* __restrict__ g, const float* __restrict__ out,
                                                        const float* __restrict__ scale,
                                                        uint16_t* __restrict__ g_heads, uint16_t* __restrict__ g_rows,
                                                        float* __restrict__ gcol_part, float* __restrict__ gsc_part,
                                                        int64_t TB, int H, int Nq, int dh) {
  const int dq4 = dh / 4;
  const int64_t B = TB * H;
  const int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= B * dq4) return;
  const int d4 = (int)(x % dq4);
  const int64_t b = x / dq4;  // = tb * H + h
  const int64_t tb = b / H;
  const int h = (int)(b - tb * H);
  const float s = __ldg(scale);
  const int n0 = blockIdx.y * kChunk;
  const int n1 = n0 + kChunk < Nq ? n0 + kChunk : Nq;
  float4 col = make_float4(0.f, 0.f, 0.f, 0.f);
  float dot = 0.0f;
  for (int n = n0; n < n1; ++n) {
    const int64_t tm = ((tb * Nq + n) * H + h) * dh + 4 * d4;  // token-major element
    const float4 gv = ld4(g + tm);
    const float4 ov = ld4(out + tm);
    dot = fmaf(gv.x, ov.x, dot);
    dot = fmaf(gv.y, ov.y, dot);
    dot = fmaf(gv.z, ov.z, dot);
    dot = fmaf(gv.w, ov.w, dot);
    const float4 gs = make_float4(gv.x * s, gv.y * s, gv.z * s, gv.w * s);
    col.x += gs.x;
    col.y += gs.y;
    col.z += gs.z;
    col.w += gs.w;
    uint2 hi, lo;
    split4(gs, hi, lo);
    uint16_t* ph = g_heads + (b * Nq + n) * (2 * dh) + 4 * d4;
    *reinterpret_cast<uint2*>(ph) = hi;
    *reinterpret_cast<uint2*>(ph + dh) = lo;
    uint16_t* pr = g_rows + ((int64_t)n * 2 * B + b) * dh + 4 * d4;
    *reinterpret_cast<uint2*>(pr) = hi;
    *reinterpret_cast<uint2*>(pr + B * dh) = lo;
  }
  *reinterpret_cast<float4*>(gcol_part + ((int64_t)blockIdx.y * B + b) * dh + 4 * d4) = col;
  gsc_part[(int64_t)blockIdx.y * B * dq4 + x] = dot;
}

template <typename OT>
__device__ __forceinline__ void store4o(OT* p, float4 v) {
  if constexpr (sizeof(OT) == 4) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    uint2 u;
    if constexpr (std::is_same<OT, __half>::value) {
      const __half2 a = __floats2half2_rn(v.x, v.y), c = __floats2half2_rn(v.z, v.w);
      u.x = *reinterpret_cast<const uint32_t*>(&a);
      u.y = *reinterpret_cast<const uint32_t*>(&c);
    } else {
      const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), c = __floats2bfloat162_rn(v.z, v.w);
      u.x = *reinterpret_cast<const uint32_t*>(&a);
      u.y = *reinterpret_cast<const uint32_t*>(&c);
    }
    *reinterpret_cast<uint2*>(p) = u;
  }
}

// head-major order over [B][Nk][dh]: dv = KE + RG[j][b] + u[b]; dk = dk32 (cast)
template <typename OT>
__global__ void __launch_bounds__(256) grad_finish_kernel(const float* __restrict__ ke, const float* __restrict__ rg,
                                                          const float* __restrict__ u, const float* __restrict__ dk32,
                                                          OT* __restrict__ dk, OT* __restrict__ dv, int64_t B, int Nk,
                                                          int dh) {
  const int dq4 = dh / 4;
  const int64_t total = B * Nk * dq4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d4 = (int)(i % dq4);
    const int64_t r = i / dq4;  // b * Nk + j
    const int j = (int)(r % Nk);
    const int64_t b = r / Nk;
    const float4 a = ld4(ke + i * 4);
    const float4 c = ld4(rg + ((int64_t)j * B + b) * dh + 4 * d4);
    const float4 e = ld4(u + b * dh + 4 * d4);
    store4o<OT>(dv + i * 4, make_float4((a.x + c.x) + e.x, (a.y + c.y) + e.y, (a.z + c.z) + e.z, (a.w + c.w) + e.w));
    store4o<OT>(dk + i * 4, ld4(dk32 + i * 4));
  }
}


// ---------------------------------------------------------------- with the output LIF

constexpr int kLifMaxT = 4;

struct LifArgs {
  const float *beta, *vth, *vr;
  float gain;
  int surrogate;
  float k, c_arctan;
};

__device__ __forceinline__ float lif_surrogate(int kind, float u, float k, float c_arctan) {
  if (kind == SPK_SURROGATE_SUPERSPIKE) {
    const float a = __fadd_rn(1.0f, __fmul_rn(k, fabsf(u)));
    return __fdiv_rn(1.0f, __fmul_rn(a, a));
  }
  const float z = __fmul_rn(c_arctan, u);
  return __fdiv_rn(__fmul_rn(k, 0.5f), __fadd_rn(1.0f, __fmul_rn(z, z)));
}

__device__ __forceinline__ void unpack4(const float* p, float* o) {
  const float4 v = ld4(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
__device__ __forceinline__ void unpack4(const __nv_bfloat16* p, float* o) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
}
__device__ __forceinline__ void unpack4(const __half* p, float* o) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
}

// one thread per (b', n, h, d4) neuron quad, all T steps: tb = t * Bp + b'
template <typename OT>
__global__ void __launch_bounds__(256) combine_lif_kernel(const float* __restrict__ qm, const float* __restrict__ rv,
                                                          const float* __restrict__ w, const float* __restrict__ scale,
                                                          LifArgs L, float* __restrict__ a_out, OT* __restrict__ spikes,
                                                          int T, int64_t Bp, int H, int Nq, int dh) {
  const int dq4 = dh / 4;
  const int64_t B = (int64_t)T * Bp * H;
  const int64_t total = Bp * Nq * H * dq4;
  const float s = __ldg(scale), beta = __ldg(L.beta), vth = __ldg(L.vth), vr = __ldg(L.vr);
  const bool use_gain = L.gain != 1.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d4 = (int)(i % dq4);
    int64_t r = i / dq4;
    const int h = (int)(r % H);
    r /= H;
    const int n = (int)(r % Nq);
    const int64_t bp = r / Nq;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int t = 0; t < T; ++t) {
      const int64_t tb = (int64_t)t * Bp + bp, b = tb * H + h;
      const float4 x = ld4(qm + (b * Nq + n) * dh + 4 * d4);
      const float4 c = ld4(rv + ((int64_t)n * B + b) * dh + 4 * d4);
      const float4 e = ld4(w + b * dh + 4 * d4);
      const float a[4] = {((x.x + c.x) + e.x) * s, ((x.y + c.y) + e.y) * s, ((x.z + c.z) + e.z) * s,
                          ((x.w + c.w) + e.w) * s};
      const int64_t tm = ((tb * Nq + n) * H + h) * dh + 4 * d4;
      *reinterpret_cast<float4*>(a_out + tm) = make_float4(a[0], a[1], a[2], a[3]);
      float sp[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float cur = use_gain ? __fmul_rn(a[q], L.gain) : a[q];
        const float u = __fadd_rn(__fmul_rn(v[q], beta), cur);
        const bool f = u > vth;
        sp[q] = f ? 1.0f : 0.0f;
        v[q] = f ? vr : u;
      }
      store4o<OT>(spikes + tm, make_float4(sp[0], sp[1], sp[2], sp[3]));
    }
  }
}

// grid: x over (b', h, d4), y over chunks of kChunk rows of n
template <typename GT>
__global__ void __launch_bounds__(256) grad_prep_lif_kernel(
    const GT* __restrict__ gsp, const float* __restrict__ a_in, const float* __restrict__ scale, LifArgs L,
    uint16_t* __restrict__ g_heads, uint16_t* __restrict__ g_rows, float* __restrict__ gcol_part,
    float* __restrict__ gsc_part, float* __restrict__ gbeta_part, int T, int64_t Bp, int H, int Nq, int dh) {
  const int dq4 = dh / 4;
  const int64_t B = (int64_t)T * Bp * H, X = Bp * H * dq4;
  const int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= X) return;
  const int d4 = (int)(x % dq4);
  const int64_t bh = x / dq4;  // = b' * H + h
  const int64_t bp = bh / H;
  const int h = (int)(bh - bp * H);
  const float s = __ldg(scale), beta = __ldg(L.beta), vth = __ldg(L.vth), vr = __ldg(L.vr);
  const bool use_gain = L.gain != 1.0f;
  const int n0 = blockIdx.y * kChunk;
  const int n1 = n0 + kChunk < Nq ? n0 + kChunk : Nq;
  float col[kLifMaxT][4];
#pragma unroll
  for (int t = 0; t < kLifMaxT; ++t)
#pragma unroll
    for (int q = 0; q < 4; ++q) col[t][q] = 0.0f;
  float dot = 0.0f, bacc = 0.0f;
  for (int n = n0; n < n1; ++n) {
    float av[kLifMaxT][4], gv[kLifMaxT][4], u[kLifMaxT][4];
    bool sb[kLifMaxT][4];
#pragma unroll
    for (int t = 0; t < kLifMaxT; ++t) {
      if (t >= T) continue;
      const int64_t tb = (int64_t)t * Bp + bp;
      const int64_t tm = ((tb * Nq + n) * H + h) * dh + 4 * d4;
      unpack4(a_in + tm, av[t]);
      unpack4(gsp + tm, gv[t]);
    }
    // membrane before reset, as the LIF forward computed it
    {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int t = 0; t < kLifMaxT; ++t) {
        if (t >= T) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float cur = use_gain ? __fmul_rn(av[t][q], L.gain) : av[t][q];
          u[t][q] = __fadd_rn(__fmul_rn(v[q], beta), cur);
          sb[t][q] = u[t][q] > vth;
          v[q] = sb[t][q] ? vr : u[t][q];
        }
      }
    }
    float gstate[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int t = kLifMaxT - 1; t >= 0; --t) {
      if (t >= T) continue;
      float gs[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float sg = lif_surrogate(L.surrogate, __fadd_rn(u[t][q], -vth), L.k, L.c_arctan);
        const float g = __fadd_rn(__fmul_rn(gv[t][q], sg), sb[t][q] ? 0.0f : gstate[q]);
        const float ga = use_gain ? __fmul_rn(g, L.gain) : g;  // dL/da
        const float vprev = t > 0 ? (sb[t - 1][q] ? vr : u[t - 1][q]) : 0.0f;
        bacc = __fadd_rn(bacc, __fmul_rn(g, vprev));
        gstate[q] = __fmul_rn(g, beta);
        dot = fmaf(ga, av[t][q], dot);
        gs[q] = ga * s;
        col[t][q] += gs[q];
      }
      const int64_t b = ((int64_t)t * Bp + bp) * H + h;
      uint2 hi, lo;
      split4(make_float4(gs[0], gs[1], gs[2], gs[3]), hi, lo);
      uint16_t* ph = g_heads + (b * Nq + n) * (2 * dh) + 4 * d4;
      *reinterpret_cast<uint2*>(ph) = hi;
      *reinterpret_cast<uint2*>(ph + dh) = lo;
      uint16_t* pr = g_rows + ((int64_t)n * 2 * B + b) * dh + 4 * d4;
      *reinterpret_cast<uint2*>(pr) = hi;
      *reinterpret_cast<uint2*>(pr + B * dh) = lo;
    }
  }
#pragma unroll
  for (int t = 0; t < kLifMaxT; ++t) {
    if (t >= T) continue;
    const int64_t b = ((int64_t)t * Bp + bp) * H + h;
    *reinterpret_cast<float4*>(gcol_part + ((int64_t)blockIdx.y * B + b) * dh + 4 * d4) =
        make_float4(col[t][0], col[t][1], col[t][2], col[t][3]);
  }
  gsc_part[(int64_t)blockIdx.y * X + x] = dot;
  if (gbeta_part) gbeta_part[(int64_t)blockIdx.y * X + x] = bacc;
}

// n_major: out[n][b][:] = in[b][n][:] for rows of r16 16-byte words (the
// n-major operand of the shared log-distance product R V).  Threads walk the
// output in order, so the stores are fully coalesced and every input row is
// read as whole 32-byte sectors.
template <typename I>
__global__ void __launch_bounds__(256) n_major_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, I B,
                                                      I N, I r16) {
  const I total = N * B * r16;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const I c = i % r16;
    const I r = i / r16;
    const I b = r % B;
    const I n = r / B;
    out[i] = __ldg(in + (b * N + n) * r16 + c);
  }
}

inline int grid_for(int64_t n4) {
  const int64_t cap = (int64_t)num_sms() * 8;
  int64_t g = (n4 + 255) / 256;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

}  // namespace xnort

static int check_dims(int64_t TB, int64_t H, int64_t N, int64_t dh) {
  SPK_REQUIRE(TB >= 1 && H >= 1 && N >= 1 && dh >= 4 && dh % 4 == 0 && TB * H * N * dh < (1ll << 40), SPK_ERR_SHAPE,
              "unsupported sizes TB=%lld H=%lld N=%lld dh=%lld (dh must be a multiple of 4)", (long long)TB,
              (long long)H, (long long)N, (long long)dh);
  return SPK_OK;
}

}  // namespace spk

extern "C" {

int spk_xnor_train_combine(const float* qm, const float* rv, const float* w, const float* scale, float* out,
                           int64_t TB, int64_t H, int64_t Nq, int64_t dh, void* stream) {
  using namespace spk;
  int rc = check_dims(TB, H, Nq, dh);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE(qm && rv && w && scale && out, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(aligned(qm, 16) && aligned(rv, 16) && aligned(w, 16) && aligned(out, 16), SPK_ERR_ALIGN,
              "qm, rv, w and out must be 16-byte aligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t n4 = TB * H * Nq * (dh / 4);
  xnort::combine_kernel<<<xnort::grid_for(n4), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      qm, rv, w, scale, out, TB, (int)H, (int)Nq, (int)dh);
  return check_launch("xnor combine_kernel");
}

int spk_xnor_train_n_major(const void* in, void* out, int64_t B, int64_t N, int64_t row_bytes, void* stream) {
  using namespace spk;
  SPK_REQUIRE(B >= 1 && N >= 1 && row_bytes >= 16 && row_bytes % 16 == 0 && B * N * row_bytes < (1ll << 40),
              SPK_ERR_SHAPE, "unsupported sizes B=%lld N=%lld row_bytes=%lld (row_bytes a multiple of 16)",
              (long long)B, (long long)N, (long long)row_bytes);
  SPK_REQUIRE(in && out, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(aligned(in, 16) && aligned(out, 16), SPK_ERR_ALIGN, "in and out must be 16-byte aligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  const int64_t r16 = row_bytes / 16, total = B * N * r16;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const auto* src = reinterpret_cast<const uint4*>(in);
  auto* dst = reinterpret_cast<uint4*>(out);
  if (total < (1ll << 30))  // 32-bit indices: total plus one grid stride stays below 2^31
    xnort::n_major_kernel<int><<<xnort::grid_for(total), 256, 0, st>>>(src, dst, (int)B, (int)N, (int)r16);
  else
    xnort::n_major_kernel<int64_t><<<xnort::grid_for(total), 256, 0, st>>>(src, dst, B, N, r16);
  return check_launch("xnor n_major_kernel");
}

int64_t spk_xnor_train_prep_chunks(int64_t Nq) { return (Nq + spk::xnort::kChunk - 1) / spk::xnort::kChunk; }

int spk_xnor_train_grad_prep(const float* g, const float* out, const float* scale, void* g_heads, void* g_rows,
                             float* gcol_part, float* gscale_part, int64_t TB, int64_t H, int64_t Nq, int64_t dh,
                             void* stream) {
  using namespace spk;
  int rc = check_dims(TB, H, Nq, dh);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE(g && out && scale && g_heads && g_rows && gcol_part && gscale_part, SPK_ERR_INVALID,
              "null pointer argument");
  SPK_REQUIRE(aligned(g, 16) && aligned(out, 16) && aligned(g_heads, 8) && aligned(g_rows, 8) &&
                  aligned(gcol_part, 16),
              SPK_ERR_ALIGN, "g, out, gcol_part must be 16-byte and g_heads, g_rows 8-byte aligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t x = TB * H * (dh / 4);
  SPK_REQUIRE((x + 255) / 256 < (1ll << 31), SPK_ERR_SHAPE, "too many heads");
  const dim3 grid((unsigned)((x + 255) / 256), (unsigned)spk_xnor_train_prep_chunks(Nq));
  SPK_REQUIRE(grid.y <= 65535, SPK_ERR_SHAPE, "Nq=%lld too long", (long long)Nq);
  xnort::grad_prep_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      g, out, scale, reinterpret_cast<uint16_t*>(g_heads), reinterpret_cast<uint16_t*>(g_rows), gcol_part, gscale_part,
      TB, (int)H, (int)Nq, (int)dh);
  return check_launch("xnor grad_prep_kernel");
}

int spk_xnor_train_grad_finish(const float* ke, const float* rg, const float* u, const float* dk32, void* dk,
                               void* dv, int out_dtype, int64_t TB, int64_t H, int64_t Nk, int64_t dh, void* stream) {
  using namespace spk;
  int rc = check_dims(TB, H, Nk, dh);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE(ke && rg && u && dk32 && dk && dv, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(out_dtype == SPK_F32 || out_dtype == SPK_F16 || out_dtype == SPK_BF16, SPK_ERR_INVALID,
              "output dtype %d not supported", out_dtype);
  SPK_REQUIRE(aligned(ke, 16) && aligned(rg, 16) && aligned(u, 16) && aligned(dk32, 16) && aligned(dk, 16) &&
                  aligned(dv, 16),
              SPK_ERR_ALIGN, "all buffers must be 16-byte aligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t B = TB * H, n4 = B * Nk * (dh / 4);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grid = xnort::grid_for(n4);
  if (out_dtype == SPK_F32)
    xnort::grad_finish_kernel<float><<<grid, 256, 0, st>>>(ke, rg, u, dk32, reinterpret_cast<float*>(dk),
                                                           reinterpret_cast<float*>(dv), B, (int)Nk, (int)dh);
  else if (out_dtype == SPK_F16)
    xnort::grad_finish_kernel<__half><<<grid, 256, 0, st>>>(ke, rg, u, dk32, reinterpret_cast<__half*>(dk),
                                                            reinterpret_cast<__half*>(dv), B, (int)Nk, (int)dh);
  else
    xnort::grad_finish_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        ke, rg, u, dk32, reinterpret_cast<__nv_bfloat16*>(dk), reinterpret_cast<__nv_bfloat16*>(dv), B, (int)Nk,
        (int)dh);
  return check_launch("xnor grad_finish_kernel");
}

int spk_xnor_train_combine_lif(const float* qm, const float* rv, const float* w, const float* scale,
                               const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                               float* a_out, void* spikes, int spike_dtype, int64_t T, int64_t TB, int64_t H,
                               int64_t Nq, int64_t dh, void* stream) {
  using namespace spk;
  int rc = check_dims(TB, H, Nq, dh);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE(T >= 1 && T <= xnort::kLifMaxT && TB % T == 0, SPK_ERR_SHAPE, "T=%lld must be in [1, %d] and divide TB=%lld",
              (long long)T, xnort::kLifMaxT, (long long)TB);
  SPK_REQUIRE(qm && rv && w && scale && lif_beta && lif_vth && lif_vreset && a_out && spikes, SPK_ERR_INVALID,
              "null pointer argument");
  SPK_REQUIRE(spike_dtype == SPK_F32 || spike_dtype == SPK_F16 || spike_dtype == SPK_BF16, SPK_ERR_INVALID,
              "spike dtype %d not supported", spike_dtype);
  SPK_REQUIRE(aligned(qm, 16) && aligned(rv, 16) && aligned(w, 16) && aligned(a_out, 16) && aligned(spikes, 16),
              SPK_ERR_ALIGN, "qm, rv, w, a_out and spikes must be 16-byte aligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t Bp = TB / T, n4 = Bp * H * Nq * (dh / 4);
  const xnort::LifArgs L{lif_beta, lif_vth, lif_vreset, in_gain, 0, 0.0f, 0.0f};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grid = xnort::grid_for(n4);
  if (spike_dtype == SPK_F32)
    xnort::combine_lif_kernel<float><<<grid, 256, 0, st>>>(qm, rv, w, scale, L, a_out, reinterpret_cast<float*>(spikes),
                                                           (int)T, Bp, (int)H, (int)Nq, (int)dh);
  else if (spike_dtype == SPK_F16)
    xnort::combine_lif_kernel<__half><<<grid, 256, 0, st>>>(qm, rv, w, scale, L, a_out,
                                                            reinterpret_cast<__half*>(spikes), (int)T, Bp, (int)H,
                                                            (int)Nq, (int)dh);
  else
    xnort::combine_lif_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(qm, rv, w, scale, L, a_out,
                                                                   reinterpret_cast<__nv_bfloat16*>(spikes), (int)T,
                                                                   Bp, (int)H, (int)Nq, (int)dh);
  return check_launch("xnor combine_lif_kernel");
}

int spk_xnor_train_grad_prep_lif(const void* g_spikes, int gs_dtype, const float* a, const float* scale,
                                 const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                                 int surrogate, float surrogate_k, void* g_heads, void* g_rows, float* gcol_part,
                                 float* gscale_part, float* gbeta_part, int64_t T, int64_t TB, int64_t H, int64_t Nq,
                                 int64_t dh, void* stream) {
  using namespace spk;
  int rc = check_dims(TB, H, Nq, dh);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE(T >= 1 && T <= xnort::kLifMaxT && TB % T == 0, SPK_ERR_SHAPE, "T=%lld must be in [1, %d] and divide TB=%lld",
              (long long)T, xnort::kLifMaxT, (long long)TB);
  SPK_REQUIRE(g_spikes && a && scale && lif_beta && lif_vth && lif_vreset && g_heads && g_rows && gcol_part &&
                  gscale_part,
              SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(gs_dtype == SPK_F32 || gs_dtype == SPK_F16 || gs_dtype == SPK_BF16, SPK_ERR_INVALID,
              "gradient dtype %d not supported", gs_dtype);
  SPK_REQUIRE(surrogate == SPK_SURROGATE_SUPERSPIKE || surrogate == SPK_SURROGATE_ARCTAN, SPK_ERR_INVALID,
              "unknown surrogate %d", surrogate);
  SPK_REQUIRE(aligned(g_spikes, 16) && aligned(a, 16) && aligned(g_heads, 8) && aligned(g_rows, 8) &&
                  aligned(gcol_part, 16),
              SPK_ERR_ALIGN, "g_spikes, a, gcol_part must be 16-byte and g_heads, g_rows 8-byte aligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t Bp = TB / T, X = Bp * H * (dh / 4);
  SPK_REQUIRE((X + 255) / 256 < (1ll << 31), SPK_ERR_SHAPE, "too many heads");
  const dim3 grid((unsigned)((X + 255) / 256), (unsigned)spk_xnor_train_prep_chunks(Nq));
  SPK_REQUIRE(grid.y <= 65535, SPK_ERR_SHAPE, "Nq=%lld too long", (long long)Nq);
  const xnort::LifArgs L{lif_beta, lif_vth, lif_vreset, in_gain, surrogate, surrogate_k,
                         (float)(3.14159265358979323846 / 2.0 * (double)surrogate_k)};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint16_t* gh = reinterpret_cast<uint16_t*>(g_heads);
  uint16_t* gr = reinterpret_cast<uint16_t*>(g_rows);
  if (gs_dtype == SPK_F32)
    xnort::grad_prep_lif_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(g_spikes), a, scale, L,
                                                             gh, gr, gcol_part, gscale_part, gbeta_part, (int)T, Bp,
                                                             (int)H, (int)Nq, (int)dh);
  else if (gs_dtype == SPK_F16)
    xnort::grad_prep_lif_kernel<__half><<<grid, 256, 0, st>>>(reinterpret_cast<const __half*>(g_spikes), a, scale,
                                                              L, gh, gr, gcol_part, gscale_part, gbeta_part, (int)T,
                                                              Bp, (int)H, (int)Nq, (int)dh);
  else
    xnort::grad_prep_lif_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(g_spikes), a, scale, L, gh, gr, gcol_part, gscale_part, gbeta_part,
        (int)T, Bp, (int)H, (int)Nq, (int)dh);
  return check_launch("xnor grad_prep_lif_kernel");
}

}  // extern "C"
