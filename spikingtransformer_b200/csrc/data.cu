// On-device training data and loss for the OCR seq2seq.
//
//   spk_synth_text_lines   synthetic text-line batch: images [B,1,H,W] fp32
//                          (U(0, 0.2) background, 5-40 black rectangles of side
//                          8-20 px per image) and uniform byte targets [B, L].
//                          Stands in for the reference's rendered Wikipedia
//                          lines (wiki_text_images3.py:173-236), which need
//                          fonts and text this build does not have; every draw
//                          comes from a counter-based hash (SplitMix64 finaliser,
//                          Steele, Lea and Flood 2014), so the batch depends only
//                          on (seed, image, draw) and a CPU restatement
//                          reproduces it bit for bit.
//   spk_ce_over_t          the training loss and metric of train_spikeformer.py:
//                          mean over the T steps of CrossEntropyLoss(ignore_index,
//                          label_smoothing) of each step's logits (:309-323,
//                          :269), and token accuracy of the argmax of the
//                          T-averaged logits over non-ignored targets (:84-93,
//                          :556-559).  One warp per (image, position) row reads
//                          the row's T x V logits once, writes dL/dlogits
//                          (before the 1 / count factor, which the caller
//                          applies) and per-block partial sums that a second
//                          kernel reduces in a fixed order.
#include "common.cuh"

namespace spk {
namespace datak {

// ---------------------------------------------------------------- counter-based draws

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// key of stream s of image b; draw i of that stream is mix64(key ^ i)
__host__ __device__ inline uint64_t stream_key(uint64_t seed, uint64_t b, uint64_t s) {
  return mix64(seed) ^ (b * 0xD1342543DE82EF95ull) ^ (s << 56);
}

__host__ __device__ inline uint64_t draw(uint64_t seed, uint64_t b, uint64_t s, uint64_t i) {
  return mix64(stream_key(seed, b, s) ^ i);
}

// uniform in [0, 1) with 24 random bits (exact in fp32)
__device__ __forceinline__ float unit24(uint64_t u) { return (float)(uint32_t)(u >> 40) * (1.0f / 16777216.0f); }

enum { S_BG = 0, S_COUNT = 1, S_RECT = 2, S_TOKEN = 3 };

// grid (pixel blocks, images); four pixels per thread and iteration, one 16-byte store
__global__ void __launch_bounds__(256) background_kernel(float* __restrict__ img, int64_t HW, uint64_t seed) {
  const int64_t b = blockIdx.y;
  const uint64_t key = stream_key(seed, (uint64_t)b, S_BG);
  float* im = img + b * HW;
  for (int64_t i = 4 * (blockIdx.x * (int64_t)blockDim.x + threadIdx.x); i < HW; i += 4 * (int64_t)gridDim.x * blockDim.x) {
    if ((HW & 3) == 0) {  // 16-byte aligned rows of 4 pixels (the image base is aligned too)
      float4 v;
      v.x = 0.2f * unit24(mix64(key ^ (uint64_t)i));
      v.y = 0.2f * unit24(mix64(key ^ (uint64_t)(i + 1)));
      v.z = 0.2f * unit24(mix64(key ^ (uint64_t)(i + 2)));
      v.w = 0.2f * unit24(mix64(key ^ (uint64_t)(i + 3)));
      *reinterpret_cast<float4*>(im + i) = v;
    } else {
      const int64_t end = i + 4 < HW ? i + 4 : HW;
      for (int64_t j = i; j < end; ++j) im[j] = 0.2f * unit24(mix64(key ^ (uint64_t)j));
    }
  }
}

// one block per image: the image's rectangles are set to 0 (black)
__global__ void __launch_bounds__(256) rectangles_kernel(float* __restrict__ img, int H, int W, uint64_t seed) {
  const int64_t b = blockIdx.x;
  float* im = img + b * (int64_t)H * W;
  const int n = 5 + (int)(draw(seed, (uint64_t)b, S_COUNT, 0) % 36ull);
  for (int r = 0; r < n; ++r) {
    const int h = 8 + (int)(draw(seed, (uint64_t)b, S_RECT, 4 * r) % 13ull);
    const int w = 8 + (int)(draw(seed, (uint64_t)b, S_RECT, 4 * r + 1) % 13ull);
    const int y = (int)(draw(seed, (uint64_t)b, S_RECT, 4 * r + 2) % (uint64_t)(H - h + 1));
    const int x = (int)(draw(seed, (uint64_t)b, S_RECT, 4 * r + 3) % (uint64_t)(W - w + 1));
    for (int k = threadIdx.x; k < h * w; k += blockDim.x) im[(int64_t)(y + k / w) * W + x + k % w] = 0.0f;
  }
}

__global__ void __launch_bounds__(256) tokens_kernel(int64_t* __restrict__ tok, int64_t B, int64_t L, int64_t V,
                                                     uint64_t seed) {
  const int64_t total = B * L;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x)
    tok[e] = (int64_t)(draw(seed, (uint64_t)(e / L), S_TOKEN, (uint64_t)(e % L)) % (uint64_t)V);
}

// ---------------------------------------------------------------- cross-entropy over T

constexpr int kCeWarps = 8;  // rows per block (one warp per row)

// part[block] = (sum of row losses over non-ignored rows, non-ignored rows, correct rows)
template <int DT, typename In = typename Elem<DT>::T>
__global__ void __launch_bounds__(32 * kCeWarps) ce_rows_kernel(const In* __restrict__ logits,
                                                                const int64_t* __restrict__ tgt, int T, int64_t rows,
                                                                int V, int64_t ignore, float eps,
                                                                In* __restrict__ grad, float* __restrict__ part,
                                                                int* __restrict__ bad) {
  __shared__ float red[kCeWarps][3];
  auto ld = [](const In* q) { return Elem<DT>::load(q); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float loss_acc = 0.0f, cnt_acc = 0.0f, cor_acc = 0.0f;
  const int64_t step = (int64_t)gridDim.x * kCeWarps;
  const int64_t tstride = rows * (int64_t)V;
  const float invT = 1.0f / (float)T;
  for (int64_t r = (int64_t)blockIdx.x * kCeWarps + warp; r < rows; r += step) {
    const int64_t y = tgt[r];
    const bool used = y != ignore;
    if (used && (y < 0 || y >= V)) {
      if (lane == 0) atomicExch(bad, 1);
    }
    const int yi = (used && y >= 0 && y < V) ? (int)y : -1;
    float row_loss = 0.0f;
    // argmax of the T-averaged logits: sum over t, then the first maximum
    float best = -INFINITY;
    int best_i = 0;
    for (int v0 = 0; v0 < V; v0 += 32) {
      const int v = v0 + lane;
      float s = -INFINITY;
      if (v < V) {
        s = 0.0f;
        for (int t = 0; t < T; ++t) s += ld(logits + t * tstride + r * V + v);
        s /= (float)T;  // the mean over the steps, as the metric takes it
      }
      if (s > best) {
        best = s;
        best_i = v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ob > best || (ob == best && oi < best_i)) {
        best = ob;
        best_i = oi;
      }
    }
    for (int t = 0; t < T; ++t) {
      const In* x = logits + t * tstride + r * V;
      // log-sum-exp (max, then sum of exp) and the sum of the logits
      float m = -INFINITY;
      for (int v = lane; v < V; v += 32) m = fmaxf(m, ld(x + v));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float se = 0.0f, sx = 0.0f;
      for (int v = lane; v < V; v += 32) {
        const float xv = ld(x + v);
        se += expf(xv - m);
        sx += xv;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
      }
      const float lse = m + logf(se);
      // loss = -(1 - eps) lp[y] - eps / V * sum_v lp[v],  lp = x - lse
      const float xy = yi >= 0 ? ld(x + yi) : 0.0f;
      row_loss += -(1.0f - eps) * (xy - lse) - eps / (float)V * (sx - (float)V * lse);
      if (grad) {
        // d/dx of this row's share of the loss, before the 1 / count factor:
        // softmax - (1 - eps) onehot - eps / V; zero for an ignored row
        In* g = grad + t * tstride + r * V;
        const float inv_se = 1.0f / se;
        for (int v = lane; v < V; v += 32) {
          const float p = expf(ld(x + v) - m) * inv_se;
          const float gv = yi >= 0 ? p - (v == yi ? 1.0f - eps : 0.0f) - eps / (float)V : 0.0f;
          g[v] = Elem<DT>::make(gv * invT);
        }
      }
    }
    if (yi >= 0) {
      loss_acc += row_loss * invT;
      cnt_acc += 1.0f;
      cor_acc += best_i == yi ? 1.0f : 0.0f;
    }
  }
  if (lane == 0) {
    red[warp][0] = loss_acc;
    red[warp][1] = cnt_acc;
    red[warp][2] = cor_acc;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float s = 0.0f;
    for (int w = 0; w < kCeWarps; ++w) s += red[w][threadIdx.x];
    part[(int64_t)blockIdx.x * 3 + threadIdx.x] = s;
  }
}

// out = (mean loss over non-ignored rows, token accuracy, 1 / max(count, 1)); fixed-order sums
__global__ void __launch_bounds__(32) ce_reduce_kernel(const float* __restrict__ part, int nblocks,
                                                       float* __restrict__ out) {
  const int lane = threadIdx.x;
  double s[3] = {0.0, 0.0, 0.0};
  for (int b = lane; b < nblocks; b += 32)
    for (int k = 0; k < 3; ++k) s[k] += (double)part[(int64_t)b * 3 + k];
  for (int k = 0; k < 3; ++k)
    for (int o = 16; o > 0; o >>= 1) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
  if (lane == 0) {
    const double cnt = s[1] > 1.0 ? s[1] : 1.0;
    out[0] = (float)(s[0] / cnt);
    out[1] = (float)(s[2] / cnt);
    out[2] = (float)(1.0 / cnt);
  }
}

inline int ce_blocks(int64_t rows) {
  int64_t need = (rows + kCeWarps - 1) / kCeWarps;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (need > cap) need = cap;
  return need < 1 ? 1 : (int)need;
}

}  // namespace datak

}  // namespace spk

extern "C" {

int spk_synth_text_lines(float* img, int64_t B, int64_t H, int64_t W, uint64_t seed, int64_t* tokens, int64_t L,
                         int64_t V, void* stream) {
  using namespace spk;
  using namespace spk::datak;
  SPK_REQUIRE(img || B == 0, SPK_ERR_INVALID, "null image buffer");
  SPK_REQUIRE(B >= 0 && H >= 20 && W >= 20 && H * W < (1ll << 40), SPK_ERR_SHAPE,
              "image size %lld x %lld unsupported (each side at least 20 px)", (long long)H, (long long)W);
  SPK_REQUIRE(!tokens || (L >= 1 && V >= 1), SPK_ERR_SHAPE, "token shape L=%lld V=%lld", (long long)L,
              (long long)V);
  SPK_REQUIRE(B < (1ll << 31), SPK_ERR_SHAPE, "too many images");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  if (B == 0) return SPK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t HW = H * W;
  SPK_REQUIRE(B < 65536, SPK_ERR_SHAPE, "at most 65535 images per call");
  SPK_REQUIRE(aligned(img, 16), SPK_ERR_ALIGN, "image buffer must be 16-byte aligned");
  int64_t per_image = (HW + 4 * 256 - 1) / (4 * 256);
  const int64_t cap = ((int64_t)num_sms() * 16 + B - 1) / B;
  if (per_image > cap) per_image = cap;
  if (per_image < 1) per_image = 1;
  background_kernel<<<dim3((unsigned)per_image, (unsigned)B), 256, 0, st>>>(img, HW, seed);
  rectangles_kernel<<<(unsigned)B, 256, 0, st>>>(img, (int)H, (int)W, seed);
  if (tokens) {
    int64_t tb = (B * L + 255) / 256;
    if (tb > (int64_t)num_sms() * 4) tb = (int64_t)num_sms() * 4;
    tokens_kernel<<<(unsigned)tb, 256, 0, st>>>(tokens, B, L, V, seed);
  }
  return check_launch("synth_text_lines");
}

int64_t spk_ce_over_t_workspace_bytes(int64_t rows) {
  return (int64_t)spk::datak::ce_blocks(rows) * 3 * (int64_t)sizeof(float);
}

int spk_ce_over_t(const void* logits, int dtype, const int64_t* targets, int64_t T, int64_t rows, int64_t V,
                  int64_t ignore_index, float label_smoothing, float* out, void* grad, void* workspace,
                  int64_t workspace_bytes, int* bad_target, void* stream) {
  using namespace spk;
  using namespace spk::datak;
  SPK_REQUIRE(logits && targets && out && bad_target, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(dtype == SPK_F32 || dtype == SPK_BF16, SPK_ERR_INVALID, "logits dtype must be fp32 or bf16");
  SPK_REQUIRE(T >= 1 && rows >= 1 && V >= 1 && V < (1 << 24) && rows * V * T < (1ll << 46), SPK_ERR_SHAPE,
              "unsupported sizes T=%lld rows=%lld V=%lld", (long long)T, (long long)rows, (long long)V);
  SPK_REQUIRE(label_smoothing >= 0.0f && label_smoothing <= 1.0f, SPK_ERR_INVALID, "label smoothing %g",
              (double)label_smoothing);
  const int nb = ce_blocks(rows);
  SPK_REQUIRE(workspace && workspace_bytes >= (int64_t)nb * 3 * 4, SPK_ERR_INVALID,
              "workspace smaller than spk_ce_over_t_workspace_bytes()");
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* part = reinterpret_cast<float*>(workspace);
  if (dtype == SPK_F32)
    ce_rows_kernel<SPK_F32><<<nb, 32 * kCeWarps, 0, st>>>(reinterpret_cast<const float*>(logits), targets, (int)T,
                                                          rows, (int)V, ignore_index, label_smoothing,
                                                          reinterpret_cast<float*>(grad), part, bad_target);
  else
    ce_rows_kernel<SPK_BF16><<<nb, 32 * kCeWarps, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits), targets, (int)T, rows, (int)V, ignore_index,
        label_smoothing, reinterpret_cast<__nv_bfloat16*>(grad), part, bad_target);
  ce_reduce_kernel<<<1, 32, 0, st>>>(part, nb, out);
  return check_launch("ce_over_t");
}

}  // extern "C"
