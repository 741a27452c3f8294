// Patch gathers (im2col) for the convolutions of the CNN image encoder.
//
// Reference: Triton_Layers/ImageEncoder.py:8-102 (CNNBackbone and its blocks:
// PixelUnshuffle + Conv2d 3x3, Conv2d 1x1, the FusedInvertedBottleneck 3x3 /
// 1x1 pair, the ReduceConvBlock 1x1 over (channel, height), the RPE2D Conv1d
// k=3).  Every one of them is a GEMM over gathered patches; the gather below
// writes those patches channels-last so that the fused tcgen05 GEMM with the
// BatchNorm-affine + LIF epilogue (spk_linear_affine_lif_fwd) consumes them.
//
// Layout: x is [N][H][W][C] (channels-last); out is [N*Ho*Wo][Kc] bf16 with
// row (n, ho, wo) and column k = (i*kw + j)*C + c for tap (i, j) of the
// kernel window; positions outside the image read 0 (zero padding).  fp32
// input is split into two bf16 terms, hi = bf16(x) in columns [0, K) and
// lo = bf16(x - hi) in [K, 2K), K = kh*kw*C, so a GEMM against [W | W]
// reproduces the fp32 convolution to about 2^-17 relative.
#include "common.cuh"

namespace spk {
namespace convk {

struct Geo {
  int64_t N;
  int H, W, C, kh, kw, sh, sw, ph, pw, Ho, Wo;
};

// bf16 input, C % 8 == 0, 16-byte aligned: one thread per 16-byte chunk
// (8 channels of one tap of one output position).
__global__ void __launch_bounds__(256) im2col_bf16_vec_kernel(const uint4* __restrict__ x, uint4* __restrict__ out,
                                                              Geo g) {
  const int cch = g.C / 8;
  const int taps = g.kh * g.kw;
  const int64_t per_row = (int64_t)taps * cch;
  const int64_t total = g.N * g.Ho * g.Wo * per_row;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / per_row;
    const int rem = (int)(e - row * per_row);
    const int tap = rem / cch, cc = rem - tap * cch;
    const int i = tap / g.kw, j = tap - i * g.kw;
    const int wo = (int)(row % g.Wo);
    const int64_t nho = row / g.Wo;
    const int ho = (int)(nho % g.Ho);
    const int64_t n = nho / g.Ho;
    const int h = ho * g.sh + i - g.ph, w = wo * g.sw + j - g.pw;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (h >= 0 && h < g.H && w >= 0 && w < g.W) v = __ldg(x + ((n * g.H + h) * g.W + w) * cch + cc);
    out[e] = v;
  }
}

// Any C: one thread per output element; fp32 input writes its hi and lo terms.
template <int XDT>
__global__ void __launch_bounds__(256) im2col_scalar_kernel(const void* __restrict__ x,
                                                            __nv_bfloat16* __restrict__ out, Geo g) {
  using XT = typename Elem<XDT>::T;
  const XT* xp = reinterpret_cast<const XT*>(x);
  const int64_t K = (int64_t)g.kh * g.kw * g.C;
  const int64_t Kc = XDT == SPK_F32 ? 2 * K : K;
  const int64_t total = g.N * g.Ho * g.Wo * K;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / K;
    const int k = (int)(e - row * K);
    const int tap = k / g.C, c = k - tap * g.C;
    const int i = tap / g.kw, j = tap - i * g.kw;
    const int wo = (int)(row % g.Wo);
    const int64_t nho = row / g.Wo;
    const int ho = (int)(nho % g.Ho);
    const int64_t n = nho / g.Ho;
    const int h = ho * g.sh + i - g.ph, w = wo * g.sw + j - g.pw;
    float v = 0.0f;
    if (h >= 0 && h < g.H && w >= 0 && w < g.W) v = Elem<XDT>::load(xp + ((n * g.H + h) * g.W + w) * g.C + c);
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    out[row * Kc + k] = hi;
    if (XDT == SPK_F32) out[row * Kc + K + k] = __float2bfloat16_rn(v - __bfloat162float(hi));
  }
}

int grid_for(int64_t items) {
  int64_t need = (items + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8 * 4;
  if (need > cap) need = cap;
  return need < 1 ? 1 : (int)need;
}

}  // namespace convk
}  // namespace spk

extern "C" {

int spk_im2col(const void* x, int x_dtype, int64_t N, int64_t H, int64_t W, int64_t C, int64_t kh, int64_t kw,
               int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, void* out, void* stream) {
  using namespace spk;
  using namespace spk::convk;
  SPK_REQUIRE(x && out, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(x_dtype == SPK_F32 || x_dtype == SPK_BF16, SPK_ERR_INVALID, "x dtype %d not supported", x_dtype);
  SPK_REQUIRE(N >= 1 && H >= 1 && W >= 1 && C >= 1 && kh >= 1 && kw >= 1 && stride_h >= 1 && stride_w >= 1 &&
                  pad_h >= 0 && pad_w >= 0 && pad_h < kh && pad_w < kw,
              SPK_ERR_SHAPE, "unsupported convolution geometry");
  SPK_REQUIRE(H + 2 * pad_h >= kh && W + 2 * pad_w >= kw, SPK_ERR_SHAPE, "kernel larger than the padded image");
  SPK_REQUIRE(H < (1 << 20) && W < (1 << 20) && C < (1 << 20) && kh * kw * C < (1 << 24), SPK_ERR_SHAPE,
              "sizes too large");
  SPK_REQUIRE(aligned(x, dtype_size(x_dtype)) && aligned(out, 2), SPK_ERR_ALIGN, "x / out misaligned");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  Geo g;
  g.N = N;
  g.H = (int)H;
  g.W = (int)W;
  g.C = (int)C;
  g.kh = (int)kh;
  g.kw = (int)kw;
  g.sh = (int)stride_h;
  g.sw = (int)stride_w;
  g.ph = (int)pad_h;
  g.pw = (int)pad_w;
  g.Ho = (int)((H + 2 * pad_h - kh) / stride_h + 1);
  g.Wo = (int)((W + 2 * pad_w - kw) / stride_w + 1);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t rows = N * g.Ho * g.Wo;
  if (x_dtype == SPK_BF16 && C % 8 == 0 && aligned(x, 16) && aligned(out, 16)) {
    const int64_t chunks = rows * kh * kw * (C / 8);
    im2col_bf16_vec_kernel<<<grid_for(chunks), 256, 0, st>>>(reinterpret_cast<const uint4*>(x),
                                                             reinterpret_cast<uint4*>(out), g);
  } else if (x_dtype == SPK_BF16) {
    im2col_scalar_kernel<SPK_BF16><<<grid_for(rows * kh * kw * C), 256, 0, st>>>(
        x, reinterpret_cast<__nv_bfloat16*>(out), g);
  } else {
    im2col_scalar_kernel<SPK_F32><<<grid_for(rows * kh * kw * C), 256, 0, st>>>(
        x, reinterpret_cast<__nv_bfloat16*>(out), g);
  }
  return check_launch("im2col kernel");
}

}  // extern "C"
