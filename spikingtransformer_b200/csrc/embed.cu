// Input-side kernels of the seq2seq forward.
//
//   spk_embed_pe_lif_fwd  TokenEmbedding (x sqrt(D)) + PositionalEncoding +
//                         T-fold + lifPE LIF, Seq2Seq.py:11-36, :109-114.
//                         The input of the LIF is the same at every step (the
//                         reference expands the embedded sequence over T,
//                         Seq2Seq.py:113), so it is computed once per element.
//   spk_patch_im2col      gathers non-overlapping p x p patches of fp32 images
//                         into GEMM rows for the patch-embedding projection,
//                         each value split into two bf16 terms (hi, lo) so a
//                         bf16 tensor-core GEMM against [W | W] reproduces the
//                         fp32 convolution to ~2^-17 relative.
#include "common.cuh"

namespace spk {
namespace embk {

template <int ODT>
__global__ void __launch_bounds__(256) embed_pe_lif_kernel(const int64_t* __restrict__ tokens,
                                                           const float* __restrict__ emb, float emb_scale,
                                                           const float* __restrict__ pe, const float* pbeta,
                                                           const float* pvth, const float* pvr, float gain, int T,
                                                           int64_t B, int64_t N, int D, int64_t V,
                                                           void* __restrict__ out, int* __restrict__ bad_token) {
  pdl_trigger();
  const float beta = __ldg(pbeta), vth = __ldg(pvth), vr = __ldg(pvr);
  pdl_wait();
  const int64_t total = B * N * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int64_t bn = i / D;
    const int64_t n = bn % N;
    int64_t tok = __ldg(tokens + bn);
    if (tok < 0 || tok >= V) {
      atomicExch(bad_token, 1);
      tok = 0;
    }
    const float x = __fadd_rn(__fmul_rn(__ldg(emb + tok * D + d), emb_scale), __ldg(pe + n * D + d));
    const float cur = gain != 1.0f ? __fmul_rn(x, gain) : x;
    float v = 0.0f;
    for (int t = 0; t < T; ++t) {
      const float u = __fadd_rn(__fmul_rn(v, beta), cur);
      const bool fire = u > vth;
      v = fire ? vr : u;
      const int64_t o = (int64_t)t * total + i;
      if (ODT == SPK_BF16)
        reinterpret_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(fire ? 1.0f : 0.0f);
      else
        reinterpret_cast<float*>(out)[o] = fire ? 1.0f : 0.0f;
    }
  }
}

// one thread per (row, c, i, j) element of the patch matrix
__global__ void __launch_bounds__(256) patch_im2col_kernel(const float* __restrict__ img, int64_t B, int C, int H,
                                                           int W, int p, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int nh = H / p, nw = W / p;
  const int K = C * p * p;
  const int64_t total = B * nh * nw * (int64_t)K;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e % K);
    const int64_t row = e / K;
    const int pw = (int)(row % nw);
    const int ph = (int)((row / nw) % nh);
    const int64_t b = row / ((int64_t)nw * nh);
    const int c = k / (p * p), ij = k % (p * p);
    const int i = ij / p, j = ij % p;
    const float x = __ldg(img + ((b * C + c) * H + (ph * p + i)) * (int64_t)W + (pw * p + j));
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
    out[row * 2 * K + k] = hi;
    out[row * 2 * K + K + k] = lo;
  }
}

// Vector form (p % 4 == 0, W % 4 == 0, 16-byte aligned image, rows < 2^31):
// a thread owns four consecutive pixels of one patch row and keeps the same
// (c, i, j4) for every patch it visits, so the per-element index arithmetic
// is one 32-bit decomposition per patch; one 16-byte load, two 8-byte stores.
__global__ void __launch_bounds__(1024) patch_im2col_vec_kernel(const float* __restrict__ img, int B, int C, int H,
                                                               int W, int p, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int nh = H / p, nw = W / p, pq = p / 4;
  const int K = C * p * p, K4 = K / 4;
  const int rows = B * nh * nw;
  const int per_block = blockDim.x / K4 > 0 ? blockDim.x / K4 : 1;  // patches side by side in one block
  const int k4 = threadIdx.x % K4, sub = threadIdx.x / K4;
  if (sub >= per_block) return;
  const int c = k4 / (p * pq), rem = k4 - c * (p * pq);
  const int i = rem / pq, j = 4 * (rem - (rem / pq) * pq);
  const int k = 4 * k4;
  for (int row = blockIdx.x * per_block + sub; row < rows; row += gridDim.x * per_block) {
    const int pw = row % nw, q = row / nw;
    const int ph = q % nh, b = q / nh;
    const float4 x = __ldg(reinterpret_cast<const float4*>(
        img + (((int64_t)b * C + c) * H + (ph * p + i)) * (int64_t)W + (pw * p + j)));
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(x.x, x.y), h1 = __floats2bfloat162_rn(x.z, x.w);
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    const __nv_bfloat162 l0 = __floats2bfloat162_rn(x.x - f0.x, x.y - f0.y);
    const __nv_bfloat162 l1 = __floats2bfloat162_rn(x.z - f1.x, x.w - f1.y);
    uint2 hv, lv;
    hv.x = *reinterpret_cast<const uint32_t*>(&h0);
    hv.y = *reinterpret_cast<const uint32_t*>(&h1);
    lv.x = *reinterpret_cast<const uint32_t*>(&l0);
    lv.y = *reinterpret_cast<const uint32_t*>(&l1);
    __nv_bfloat16* o = out + (int64_t)row * 2 * K + k;
    *reinterpret_cast<uint2*>(o) = hv;
    *reinterpret_cast<uint2*>(o + K) = lv;
  }
}

}  // namespace embk

static int grid_1d(int64_t n) {
  int64_t g = (n + 255) / 256;
  int64_t cap = (int64_t)num_sms() * 32;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace spk

extern "C" {

int spk_embed_pe_lif_fwd(const int64_t* tokens, const float* emb, float emb_scale, const float* pe,
                         const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                         int64_t T, int64_t B, int64_t N, int64_t D, int64_t V, void* out, int out_dtype,
                         int* bad_token, void* stream) {
  using namespace spk;
  SPK_REQUIRE(tokens && emb && pe && lif_beta && lif_vth && lif_vreset && out && bad_token, SPK_ERR_INVALID,
              "null pointer argument");
  SPK_REQUIRE(out_dtype == SPK_BF16 || out_dtype == SPK_F32, SPK_ERR_INVALID, "out dtype must be bf16 or f32");
  SPK_REQUIRE(T >= 1 && T <= 1024 && B >= 0 && N >= 0 && D >= 1 && D < (1 << 24) && V >= 1, SPK_ERR_SHAPE,
              "unsupported sizes");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  if (B * N == 0) return SPK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_1d(B * N * D), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  add_pdl_attr(cfg, attr);
  const int iT = (int)T, iD = (int)D;
  const cudaError_t e =
      out_dtype == SPK_BF16
          ? cudaLaunchKernelEx(&cfg, embk::embed_pe_lif_kernel<SPK_BF16>, tokens, emb, emb_scale, pe, lif_beta,
                               lif_vth, lif_vreset, in_gain, iT, B, N, iD, V, out, bad_token)
          : cudaLaunchKernelEx(&cfg, embk::embed_pe_lif_kernel<SPK_F32>, tokens, emb, emb_scale, pe, lif_beta,
                               lif_vth, lif_vreset, in_gain, iT, B, N, iD, V, out, bad_token);
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "embed_pe_lif_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

int spk_patch_im2col(const float* img, int64_t B, int64_t C, int64_t H, int64_t W, int64_t patch, void* out,
                     void* stream) {
  using namespace spk;
  SPK_REQUIRE(img && out, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(patch >= 1 && C >= 1 && H % patch == 0 && W % patch == 0 && B >= 0, SPK_ERR_SHAPE,
              "image %lldx%lld not divisible into %lld-pixel patches", (long long)H, (long long)W, (long long)patch);
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  if (B == 0) return SPK_OK;
  const int64_t n = B * (H / patch) * (W / patch) * C * patch * patch;
  const int64_t rows = B * (H / patch) * (W / patch);
  const int64_t K4 = C * patch * patch / 4;
  if (patch % 4 == 0 && W % 4 == 0 && aligned(img, 16) && aligned(out, 8) && rows < (1ll << 31) && K4 <= 1024 &&
      B * C * H * W < (1ll << 40)) {
    cudaLaunchConfig_t cv = {};
    const int threads = K4 >= 256 ? (int)K4 : (int)(256 / K4 * K4);
    const int per_block = threads / (int)K4;
    int64_t g = (rows + per_block - 1) / per_block;
    const int64_t cap = (int64_t)num_sms() * (2048 / threads);
    if (g > cap) g = cap;
    cv.gridDim = dim3((unsigned)(g < 1 ? 1 : g), 1, 1);
    cv.blockDim = dim3((unsigned)threads, 1, 1);
    cv.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute av[1];
    add_pdl_attr(cv, av);
    const cudaError_t e = cudaLaunchKernelEx(&cv, embk::patch_im2col_vec_kernel, img, (int)B, (int)C, (int)H, (int)W,
                                             (int)patch, reinterpret_cast<__nv_bfloat16*>(out));
    if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "patch_im2col_vec_kernel launch: %s", cudaGetErrorString(e));
    return SPK_OK;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid_1d(n), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  add_pdl_attr(cfg, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, embk::patch_im2col_kernel, img, B, (int)C, (int)H, (int)W,
                                           (int)patch, reinterpret_cast<__nv_bfloat16*>(out));
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "patch_im2col_kernel launch: %s", cudaGetErrorString(e));
  return SPK_OK;
}

}  // extern "C"
