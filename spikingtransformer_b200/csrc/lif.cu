// LIF temporal scan, forward and backward (HBM-bound elementwise recurrences).
//
// Reference: Triton_Layers/Lif.py:118-165 (forward), :181-282 (backward).
// Layout: x, spikes, grads are [T][N] (N = batch * features, t-major), the
// reference's [T, B, F] after .contiguous().
//
// One thread owns VEC consecutive neurons and walks all T steps with the
// membrane in registers; loads and stores are 16-byte vectors where the
// pointers allow.  The backward keeps the pre-reset membrane of all T steps in
// registers (T <= 64), so unlike the reference there is no v_mem_history
// round trip through HBM.  Arithmetic uses explicitly rounded fp32 operations
// (__fmul_rn / __fadd_rn / __fdiv_rn, never contracted into FMA) in the
// reference's order, so results are bit-identical to the reference evaluated
// in fp32 one operation at a time.
#include <mutex>

#include "common.cuh"

namespace spk {
namespace lifk {

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC >= 16 ? 16 : sizeof(T) * VEC) Pack {
  T v[VEC];
};

template <int DT, int VEC>
__device__ __forceinline__ void load_vec(const void* base, int64_t idx, float* out) {
  using T = typename Elem<DT>::T;
  const T* p = reinterpret_cast<const T*>(base) + idx;
  if constexpr (VEC == 1) {
    out[0] = Elem<DT>::load(p);
  } else if constexpr (sizeof(T) * VEC <= 16) {
    Pack<T, VEC> pk = *reinterpret_cast<const Pack<T, VEC>*>(p);
#pragma unroll
    for (int i = 0; i < VEC; ++i) out[i] = Elem<DT>::load(&pk.v[i]);
  } else {
    constexpr int H = VEC / 2;
    load_vec<DT, H>(base, idx, out);
    load_vec<DT, H>(base, idx + H, out + H);
  }
}

template <int DT, int VEC>
__device__ __forceinline__ void store_vec(void* base, int64_t idx, const float* in) {
  using T = typename Elem<DT>::T;
  T* p = reinterpret_cast<T*>(base) + idx;
  if constexpr (VEC == 1) {
    *p = Elem<DT>::make(in[0]);
  } else if constexpr (sizeof(T) * VEC <= 16) {
    Pack<T, VEC> pk;
#pragma unroll
    for (int i = 0; i < VEC; ++i) pk.v[i] = Elem<DT>::make(in[i]);
    *reinterpret_cast<Pack<T, VEC>*>(p) = pk;
  } else {
    constexpr int H = VEC / 2;
    store_vec<DT, H>(base, idx, in);
    store_vec<DT, H>(base, idx + H, in + H);
  }
}

template <int XDT, int SDT, int VEC>
__global__ void __launch_bounds__(256) lif_fwd_kernel(const void* __restrict__ x, void* __restrict__ spikes,
                                                      float* __restrict__ v_final, const float* pbeta,
                                                      const float* pvth, const float* pvr, float gain, int T,
                                                      int64_t N) {
  const float beta = __ldg(pbeta), vth = __ldg(pvth), vr = __ldg(pvr);
  const bool use_gain = gain != 1.0f;
  const int64_t groups = N / VEC;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    float v[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = 0.0f;
    const int64_t col = g * VEC;
    for (int t = 0; t < T; ++t) {
      float xv[VEC], sv[VEC];
      load_vec<XDT, VEC>(x, (int64_t)t * N + col, xv);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        float cur = use_gain ? __fmul_rn(xv[i], gain) : xv[i];
        float u = __fadd_rn(__fmul_rn(v[i], beta), cur);
        bool s = u > vth;
        sv[i] = s ? 1.0f : 0.0f;
        v[i] = s ? vr : u;
      }
      store_vec<SDT, VEC>(spikes, (int64_t)t * N + col, sv);
    }
    if (v_final) store_vec<SPK_F32, VEC>(v_final, col, v);
  }
}

// Packed-bit spikes: thread g owns neurons [8g, 8g + 8) and writes one byte
// per step, bit i for neuron 8g + i, into rows of ceil(N/8) bytes; a warp's
// stores cover 32 consecutive bytes.  `vec`: N % 8 == 0 and x aligned for
// 8-element vector loads; otherwise elements are loaded one by one with a
// bound on the last group.
template <int XDT>
__global__ void __launch_bounds__(256) lif_fwd_bits_kernel(const void* __restrict__ x, uint8_t* __restrict__ spikes,
                                                           float* __restrict__ v_final, const float* pbeta,
                                                           const float* pvth, const float* pvr, float gain, int T,
                                                           int64_t N, bool vec) {
  using XT = typename Elem<XDT>::T;
  const float beta = __ldg(pbeta), vth = __ldg(pvth), vr = __ldg(pvr);
  const bool use_gain = gain != 1.0f;
  const int64_t NB = (N + 7) / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < NB; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = g * 8;
    const int n = N - col < 8 ? (int)(N - col) : 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    for (int t = 0; t < T; ++t) {
      float xv[8];
      if (vec) {
        load_vec<XDT, 8>(x, (int64_t)t * N + col, xv);
      } else {
        const XT* row = reinterpret_cast<const XT*>(x) + (int64_t)t * N + col;
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[i] = i < n ? Elem<XDT>::load(row + i) : 0.0f;
      }
      uint32_t bits = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float cur = use_gain ? __fmul_rn(xv[i], gain) : xv[i];
        float u = __fadd_rn(__fmul_rn(v[i], beta), cur);
        bool s = u > vth && i < n;
        bits |= (s ? 1u : 0u) << i;
        v[i] = s ? vr : u;
      }
      spikes[(int64_t)t * NB + g] = (uint8_t)bits;
    }
    if (v_final) {
      if (vec) {
        store_vec<SPK_F32, 8>(v_final, col, v);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < n) v_final[col + i] = v[i];
      }
    }
  }
}

// Spike bits of neurons [col, col + VEC) at step t (bit i = neuron col + i).
template <int SDT, int VEC>
__device__ __forceinline__ uint32_t load_spike_bits(const void* spikes, int t, int64_t N, int64_t col) {
  if constexpr (SDT == SPK_BIT) {
    static_assert(VEC == 1 || VEC == 4, "packed bits are read 1 or 4 at a time");
    const uint8_t* row = reinterpret_cast<const uint8_t*>(spikes) + (int64_t)t * ((N + 7) / 8);
    const uint32_t byte = __ldg(row + (col >> 3));
    return (byte >> (col & 7)) & ((1u << VEC) - 1u);
  } else {
    float sv[VEC];
    load_vec<SDT, VEC>(spikes, (int64_t)t * N + col, sv);
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < VEC; ++i) bits |= (sv[i] > 0.0f ? 1u : 0u) << i;
    return bits;
  }
}

__device__ __forceinline__ float surrogate(int kind, float u, float k, float c_arctan) {
  if (kind == SPK_SURROGATE_SUPERSPIKE) {
    float a = __fadd_rn(1.0f, __fmul_rn(k, fabsf(u)));
    return __fdiv_rn(__fdiv_rn(1.0f, a), a);
  }
  float z = __fmul_rn(c_arctan, u);
  return __fdiv_rn(__fmul_rn(k, 0.5f), __fadd_rn(1.0f, __fmul_rn(z, z)));
}

constexpr int kBwdThreads = 256;
constexpr int kBwdMaxBlocks = 4096;

template <int XDT, int SDT, int TMAX, int VEC>
__global__ void __launch_bounds__(kBwdThreads, TMAX <= 4 ? 3 : 1) lif_bwd_kernel(
    const float* __restrict__ gs, const float* __restrict__ gvf, const void* __restrict__ x,
    const void* __restrict__ spikes, const float* pbeta, const float* pvth, const float* pvr, float gain,
    int surr, float k, float c_arctan, void* __restrict__ gx, float* __restrict__ partials, int T, int64_t N) {
  const float beta = __ldg(pbeta), vth = __ldg(pvth), vr = __ldg(pvr);
  const bool use_gain = gain != 1.0f;
  const int64_t groups = N / VEC;
  float thread_acc = 0.0f;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = g * VEC;
    float vh[TMAX][VEC];
    uint32_t sbits[TMAX];
    float v[VEC];
    // short scans (T <= 4) load the spike gradients of every step up front,
    // beside the inputs, so a thread's loads are all in flight at once
    constexpr bool kPreload = TMAX <= 4;
    float gpre[kPreload ? TMAX : 1][VEC];
    if constexpr (kPreload) {
#pragma unroll
      for (int t = 0; t < TMAX; ++t)
        if (t < T) load_vec<SPK_F32, VEC>(gs, (int64_t)t * N + col, gpre[t]);
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = 0.0f;
    // pass 1: recompute the pre-reset membrane (Lif.py:222-233)
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
      if (t < T) {
        float xv[VEC];
        load_vec<XDT, VEC>(x, (int64_t)t * N + col, xv);
        const uint32_t bits = load_spike_bits<SDT, VEC>(spikes, t, N, col);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          float cur = use_gain ? __fmul_rn(xv[i], gain) : xv[i];
          float u = __fadd_rn(__fmul_rn(v[i], beta), cur);
          vh[t][i] = u;
          v[i] = ((bits >> i) & 1u) ? vr : u;
        }
        sbits[t] = bits;
      }
    }
    // pass 2: reverse sweep (Lif.py:236-273)
    float gstate[VEC], acc[VEC];
    if (gvf) {
      load_vec<SPK_F32, VEC>(gvf, col, gstate);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) gstate[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
#pragma unroll
    for (int t = TMAX - 1; t >= 0; --t) {
      if (t < T) {
        float gsv[VEC], out[VEC];
        if constexpr (kPreload) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) gsv[i] = gpre[kPreload ? t : 0][i];
        } else {
          load_vec<SPK_F32, VEC>(gs, (int64_t)t * N + col, gsv);
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const bool s = (sbits[t] >> i) & 1u;
          const float sg = surrogate(surr, __fadd_rn(vh[t][i], -vth), k, c_arctan);
          const float from_state = s ? 0.0f : gstate[i];
          const float gv = __fadd_rn(__fmul_rn(gsv[i], sg), from_state);
          out[i] = use_gain ? __fmul_rn(gv, gain) : gv;
          float vprev = 0.0f;
          if (t > 0) vprev = ((sbits[t - 1] >> i) & 1u) ? vr : vh[t - 1][i];
          acc[i] = __fadd_rn(acc[i], __fmul_rn(gv, vprev));
          gstate[i] = __fmul_rn(gv, beta);
        }
        store_vec<XDT, VEC>(gx, (int64_t)t * N + col, out);
      }
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) thread_acc += acc[i];
  }
  // deterministic block reduction of the grad_beta partial
  __shared__ float red[kBwdThreads / 32];
  float s = thread_acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < kBwdThreads / 32 ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0 && partials) partials[blockIdx.x] = r;
  }
}

// ---- backward, staged through shared memory (fp32 x, T <= 4) --------------
// Persistent blocks walk tiles of kSTile neurons.  One thread issues bulk
// copies (cp.async.bulk, contiguous rows, no tensor map) of a tile's x,
// spike-gradient, spike and g_vfinal rows into a ring of shared-memory stages,
// up to kSStages tiles ahead, so the loads of the next tiles are in flight
// while a tile is computed and no registers are spent holding them.  The
// arithmetic is the register kernel's, operation for operation, so the
// results are the same bit for bit.
constexpr int kSTile = 4 * kBwdThreads;  // neurons per tile (4 per thread)
constexpr int kSRow = kSTile * 4;        // bytes of one fp32 row of a tile

template <int SDT>
__host__ __device__ constexpr int staged_spike_row(int n) {
  return SDT == SPK_BIT ? n / 8 : SDT == SPK_BF16 ? 2 * n : n;
}
template <int SDT>
__host__ __device__ constexpr int staged_stages() {
  return SDT == SPK_BIT ? 3 : 2;
}
// stage: x [4][kSTile] f32 | g_s [4][kSTile] f32 | g_vfinal [kSTile] f32 | spikes [4][row]
template <int SDT>
__host__ __device__ constexpr int staged_stage_bytes() {
  return (9 * kSRow + 4 * staged_spike_row<SDT>(kSTile) + 127) / 128 * 128;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int SDT>
__global__ void __launch_bounds__(kBwdThreads, 2) lif_bwd_staged_kernel(
    const float* __restrict__ gs, const float* __restrict__ gvf, const float* __restrict__ x,
    const void* __restrict__ spikes, const float* pbeta, const float* pvth, const float* pvr, float gain,
    int surr, float k, float c_arctan, float* __restrict__ gx, float* __restrict__ partials, int T, int64_t N) {
  constexpr int S = staged_stages<SDT>();
  constexpr int SB = staged_spike_row<SDT>(kSTile);
  constexpr int kStage = staged_stage_bytes<SDT>();
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[S];
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int64_t tiles = (N + kSTile - 1) / kSTile;
  const int my = (int)((tiles - (int64_t)blockIdx.x + gridDim.x - 1) / gridDim.x);
  const int64_t srow = SDT == SPK_BIT ? N / 8 : (int64_t)staged_spike_row<SDT>(1) * N;  // spike bytes per step
  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const float beta = __ldg(pbeta), vth = __ldg(pvth), vr = __ldg(pvr);
  const bool use_gain = gain != 1.0f;
  // tile j of this block's sequence into stage j % S
  auto issue = [&](int j) {
    const int s = j % S;
    const int64_t base = ((int64_t)blockIdx.x + (int64_t)j * gridDim.x) * kSTile;
    const int64_t left = N - base;
    const int n = left < kSTile ? (int)left : kSTile;
    const uint32_t rb = (uint32_t)n * 4u, sb = (uint32_t)staged_spike_row<SDT>(n);
    const int64_t sbase = SDT == SPK_BIT ? base / 8 : base * staged_spike_row<SDT>(1);  // spike bytes before the tile
    uint8_t* st = smem + (size_t)s * kStage;
    mbar_expect_tx(&full[s], (uint32_t)T * (2u * rb + sb) + (gvf ? rb : 0u));
    for (int t = 0; t < T; ++t) {
      bulk_load(st + t * kSRow, x + (int64_t)t * N + base, rb, &full[s]);
      bulk_load(st + (4 + t) * kSRow, gs + (int64_t)t * N + base, rb, &full[s]);
      bulk_load(st + 9 * kSRow + t * SB, reinterpret_cast<const uint8_t*>(spikes) + t * srow + sbase, sb, &full[s]);
    }
    if (gvf) bulk_load(st + 8 * kSRow, gvf + base, rb, &full[s]);
  };
  if (tid == 0)
    for (int j = 0; j < S && j < my; ++j) issue(j);
  float thread_acc = 0.0f;
  int j = 0;
  for (; j < my; ++j) {
    const int s = j % S;
    if (!mbar_wait(&full[s], (uint32_t)(j / S) & 1u, 181)) abort_flag = 1;
    const int64_t base = ((int64_t)blockIdx.x + (int64_t)j * gridDim.x) * kSTile;
    const int64_t left = N - base;
    const int n = left < kSTile ? (int)left : kSTile;
    const uint8_t* st = smem + (size_t)s * kStage;
    if (!abort_flag && tid * 4 < n) {
      const int col = tid * 4;
      float vh[4][4], gsv[4][4], v[4];
      uint32_t sbits[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (t < T) {
          const float4 g4 = *reinterpret_cast<const float4*>(st + (4 + t) * kSRow + col * 4);
          gsv[t][0] = g4.x; gsv[t][1] = g4.y; gsv[t][2] = g4.z; gsv[t][3] = g4.w;
          if constexpr (SDT == SPK_BIT) {
            const uint32_t byte = st[9 * kSRow + t * SB + (col >> 3)];
            sbits[t] = (byte >> (col & 7)) & 0xFu;
          } else {
            float sv[4];
            load_vec<SDT, 4>(st + 9 * kSRow + t * SB, col, sv);
            uint32_t bits = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) bits |= (sv[i] > 0.0f ? 1u : 0u) << i;
            sbits[t] = bits;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = 0.0f;
      // pass 1: the pre-reset membrane (Lif.py:222-233)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (t < T) {
          const float4 x4 = *reinterpret_cast<const float4*>(st + t * kSRow + col * 4);
          const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float cur = use_gain ? __fmul_rn(xv[i], gain) : xv[i];
            float u = __fadd_rn(__fmul_rn(v[i], beta), cur);
            vh[t][i] = u;
            v[i] = ((sbits[t] >> i) & 1u) ? vr : u;
          }
        }
      }
      // pass 2: reverse sweep (Lif.py:236-273)
      float gstate[4], acc[4];
      if (gvf) {
        const float4 v4 = *reinterpret_cast<const float4*>(st + 8 * kSRow + col * 4);
        gstate[0] = v4.x; gstate[1] = v4.y; gstate[2] = v4.z; gstate[3] = v4.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) gstate[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int t = 3; t >= 0; --t) {
        if (t < T) {
          float out[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool sp = (sbits[t] >> i) & 1u;
            const float sg = surrogate(surr, __fadd_rn(vh[t][i], -vth), k, c_arctan);
            const float from_state = sp ? 0.0f : gstate[i];
            const float gv = __fadd_rn(__fmul_rn(gsv[t][i], sg), from_state);
            out[i] = use_gain ? __fmul_rn(gv, gain) : gv;
            float vprev = 0.0f;
            if (t > 0) vprev = ((sbits[t - 1] >> i) & 1u) ? vr : vh[t - 1][i];
            acc[i] = __fadd_rn(acc[i], __fmul_rn(gv, vprev));
            gstate[i] = __fmul_rn(gv, beta);
          }
          *reinterpret_cast<float4*>(gx + (int64_t)t * N + base + col) = make_float4(out[0], out[1], out[2], out[3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) thread_acc += acc[i];
    }
    __syncthreads();  // every thread is done with stage s (and has seen abort_flag)
    if (abort_flag) break;
    if (tid == 0 && j + S < my) {
      fence_proxy_async_smem();  // the reads above come before the copies that overwrite them
      issue(j + S);
    }
  }
  if (abort_flag && tid == 0) {
    // tiles j .. j + S - 1 may still have copies in flight: let them land
    // before the block exits (each wait bounded)
    for (int jj = j; jj < my && jj < j + S; ++jj) mbar_wait(&full[jj % S], (uint32_t)(jj / S) & 1u, 182);
  }
  // deterministic block reduction of the grad_beta partial
  __shared__ float red[kBwdThreads / 32];
  float s = thread_acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < kBwdThreads / 32 ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0 && partials) partials[blockIdx.x] = r;
  }
}

__global__ void __launch_bounds__(1024) sum_partials_kernel(const float* __restrict__ partials, int n,
                                                            float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < (int)(blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0) *out = r;
  }
}

int grid_for(int64_t groups, int threads) {
  int64_t need = (groups + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * (2048 / threads) * 4;
  if (need > cap) need = cap;
  if (need < 1) need = 1;
  return (int)need;
}

template <int XDT, int SDT, int VEC>
void launch_fwd(const void* x, void* s, float* vf, const float* b, const float* th, const float* vr, float gain,
                int T, int64_t N, cudaStream_t st) {
  int grid = grid_for(N / VEC, 256);
  lif_fwd_kernel<XDT, SDT, VEC><<<grid, 256, 0, st>>>(x, s, vf, b, th, vr, gain, T, N);
}

template <int XDT, int SDT>
void dispatch_fwd_vec(bool vec, const void* x, void* s, float* vf, const float* b, const float* th,
                      const float* vr, float gain, int T, int64_t N, cudaStream_t st) {
  if (vec)
    launch_fwd<XDT, SDT, 8>(x, s, vf, b, th, vr, gain, T, N, st);
  else
    launch_fwd<XDT, SDT, 1>(x, s, vf, b, th, vr, gain, T, N, st);
}

template <int XDT>
int dispatch_fwd_s(int sdt, bool vec, const void* x, void* s, float* vf, const float* b, const float* th,
                   const float* vr, float gain, int T, int64_t N, cudaStream_t st) {
  switch (sdt) {
    case SPK_F32: dispatch_fwd_vec<XDT, SPK_F32>(vec, x, s, vf, b, th, vr, gain, T, N, st); return SPK_OK;
    case SPK_BF16: dispatch_fwd_vec<XDT, SPK_BF16>(vec, x, s, vf, b, th, vr, gain, T, N, st); return SPK_OK;
    case SPK_U8: dispatch_fwd_vec<XDT, SPK_U8>(vec, x, s, vf, b, th, vr, gain, T, N, st); return SPK_OK;
    case SPK_FP8: dispatch_fwd_vec<XDT, SPK_FP8>(vec, x, s, vf, b, th, vr, gain, T, N, st); return SPK_OK;
    case SPK_BIT: {
      int grid = grid_for((N + 7) / 8, 256);
      lif_fwd_bits_kernel<XDT><<<grid, 256, 0, st>>>(x, reinterpret_cast<uint8_t*>(s), vf, b, th, vr, gain, T, N,
                                                     vec);
      return SPK_OK;
    }
    default: return fail(SPK_ERR_INVALID, "spike dtype %d not supported", sdt);
  }
}

template <int XDT, int SDT, int TMAX, int VEC>
void launch_bwd(int grid, const float* gs, const float* gvf, const void* x, const void* s, const float* b,
                const float* th, const float* vr, float gain, int surr, float k, float c, void* gx, float* part,
                int T, int64_t N, cudaStream_t st) {
  lif_bwd_kernel<XDT, SDT, TMAX, VEC><<<grid, kBwdThreads, 0, st>>>(gs, gvf, x, s, b, th, vr, gain, surr, k, c,
                                                                    gx, part, T, N);
}

// The staged backward for fp32 x and T <= 4; returns the grid it launched
// (the number of grad_beta partials), or 0 when it does not take the call.
template <int SDT>
int launch_bwd_staged(const float* gs, const float* gvf, const float* x, const void* s, const float* b,
                      const float* th, const float* vr, float gain, int surr, float k, float c, float* gx,
                      float* part, int T, int64_t N, cudaStream_t st) {
  const int64_t tiles = (N + kSTile - 1) / kSTile;
  int64_t grid = 2 * (int64_t)num_sms();
  if (grid > tiles) grid = tiles;
  const int smem = staged_stages<SDT>() * staged_stage_bytes<SDT>();
  if (cudaFuncSetAttribute(lif_bwd_staged_kernel<SDT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return 0;
  lif_bwd_staged_kernel<SDT><<<(int)grid, kBwdThreads, smem, st>>>(gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx,
                                                                    part, T, N);
  return (int)grid;
}

template <int XDT, int SDT>
int dispatch_bwd_t(int T, bool vec, int grid, const float* gs, const float* gvf, const void* x, const void* s,
                   const float* b, const float* th, const float* vr, float gain, int surr, float k, float c,
                   void* gx, float* part, int64_t N, cudaStream_t st) {
  if (T <= 4) {
    if (vec) launch_bwd<XDT, SDT, 4, 4>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
    else launch_bwd<XDT, SDT, 4, 1>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
  } else if (T <= 8) {
    if (vec) launch_bwd<XDT, SDT, 8, 4>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
    else launch_bwd<XDT, SDT, 8, 1>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
  } else if (T <= 16) {
    if (vec) launch_bwd<XDT, SDT, 16, 4>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
    else launch_bwd<XDT, SDT, 16, 1>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
  } else {
    launch_bwd<XDT, SDT, 64, 1>(grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, T, N, st);
  }
  return SPK_OK;
}

template <int XDT>
int dispatch_bwd_s(int sdt, int T, bool vec, int grid, const float* gs, const float* gvf, const void* x,
                   const void* s, const float* b, const float* th, const float* vr, float gain, int surr, float k,
                   float c, void* gx, float* part, int64_t N, cudaStream_t st) {
  switch (sdt) {
    case SPK_F32:
      return dispatch_bwd_t<XDT, SPK_F32>(T, vec, grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, N, st);
    case SPK_BF16:
      return dispatch_bwd_t<XDT, SPK_BF16>(T, vec, grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, N, st);
    case SPK_U8:
      return dispatch_bwd_t<XDT, SPK_U8>(T, vec, grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, N, st);
    case SPK_FP8:
      return dispatch_bwd_t<XDT, SPK_FP8>(T, vec, grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, N, st);
    case SPK_BIT:
      return dispatch_bwd_t<XDT, SPK_BIT>(T, vec, grid, gs, gvf, x, s, b, th, vr, gain, surr, k, c, gx, part, N, st);
    default: return fail(SPK_ERR_INVALID, "spike dtype %d not supported", sdt);
  }
}

}  // namespace lifk

using namespace lifk;

SPK_DEFINE_ERROR_READER(lif_read_device_error)

// Shared implementation of the backward entry points: `partials` holds at
// least bwd_grid(T, N) floats.
int lif_bwd_impl(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype, const void* spikes,
                 int spike_dtype, const float* beta, const float* v_th, const float* v_reset, float in_gain,
                 int surrogate_kind, float surrogate_k, void* grad_x, float* grad_beta, float* partials,
                 int64_t T, int64_t N, cudaStream_t st);

int lif_bwd_grid(int64_t T, int64_t N) {
  const bool vec = true;
  int64_t groups = vec && T <= 16 ? N / 4 : N;
  int g = grid_for(groups, kBwdThreads);
  return g > kBwdMaxBlocks ? kBwdMaxBlocks : g;
}

int lif_bwd_impl(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype, const void* spikes,
                 int spike_dtype, const float* beta, const float* v_th, const float* v_reset, float in_gain,
                 int surrogate_kind, float surrogate_k, void* grad_x, float* grad_beta, float* partials,
                 int64_t T, int64_t N, cudaStream_t st) {
  // the vector path needs N % 4 == 0 and 16-byte aligned rows for fp32 tensors
  bool vec = T <= 16 && (N % 4 == 0) && aligned(g_spikes, 16) && (!g_vfinal || aligned(g_vfinal, 16)) &&
             aligned(x, 4 * dtype_size(x_dtype)) &&
             (spike_dtype == SPK_BIT || aligned(spikes, 4 * dtype_size(spike_dtype))) &&
             aligned(grad_x, 4 * dtype_size(x_dtype));
  int64_t groups = vec ? N / 4 : N;
  int grid = grid_for(groups, kBwdThreads);
  if (grid > kBwdMaxBlocks) grid = kBwdMaxBlocks;
  const float c = (float)(3.14159265358979323846 / 2.0 * (double)surrogate_k);
  int rc;
  // fp32 currents, T <= 4, whole 128-neuron blocks and 16-byte aligned rows:
  // the kernel that stages its inputs through shared memory with bulk copies
  const bool staged = x_dtype == SPK_F32 && T <= 4 && N > 0 && N % 128 == 0 &&
                      (spike_dtype == SPK_BIT || spike_dtype == SPK_BF16 || spike_dtype == SPK_U8 ||
                       spike_dtype == SPK_FP8) &&
                      aligned(g_spikes, 16) && (!g_vfinal || aligned(g_vfinal, 16)) && aligned(x, 16) &&
                      aligned(spikes, 16) && aligned(grad_x, 16);
  if (staged) {
    const float* xf = static_cast<const float*>(x);
    float* gxf = static_cast<float*>(grad_x);
    int sg = 0;
    switch (spike_dtype) {
      case SPK_BIT: sg = launch_bwd_staged<SPK_BIT>(g_spikes, g_vfinal, xf, spikes, beta, v_th, v_reset, in_gain, surrogate_kind, surrogate_k, c, gxf, partials, (int)T, N, st); break;
      case SPK_BF16: sg = launch_bwd_staged<SPK_BF16>(g_spikes, g_vfinal, xf, spikes, beta, v_th, v_reset, in_gain, surrogate_kind, surrogate_k, c, gxf, partials, (int)T, N, st); break;
      case SPK_U8: sg = launch_bwd_staged<SPK_U8>(g_spikes, g_vfinal, xf, spikes, beta, v_th, v_reset, in_gain, surrogate_kind, surrogate_k, c, gxf, partials, (int)T, N, st); break;
      default: sg = launch_bwd_staged<SPK_FP8>(g_spikes, g_vfinal, xf, spikes, beta, v_th, v_reset, in_gain, surrogate_kind, surrogate_k, c, gxf, partials, (int)T, N, st); break;
    }
    if (sg > 0) {
      if ((rc = check_launch("lif_bwd_staged_kernel")) != SPK_OK) return rc;
      if (grad_beta) {
        sum_partials_kernel<<<1, 1024, 0, st>>>(partials, sg, grad_beta);
        if ((rc = check_launch("sum_partials_kernel")) != SPK_OK) return rc;
      }
      return SPK_OK;
    }
  }
  switch (x_dtype) {
    case SPK_F32:
      rc = dispatch_bwd_s<SPK_F32>(spike_dtype, (int)T, vec, grid, g_spikes, g_vfinal, x, spikes, beta, v_th,
                                   v_reset, in_gain, surrogate_kind, surrogate_k, c, grad_x, partials, N, st);
      break;
    case SPK_F16:
      rc = dispatch_bwd_s<SPK_F16>(spike_dtype, (int)T, vec, grid, g_spikes, g_vfinal, x, spikes, beta, v_th,
                                   v_reset, in_gain, surrogate_kind, surrogate_k, c, grad_x, partials, N, st);
      break;
    case SPK_BF16:
      rc = dispatch_bwd_s<SPK_BF16>(spike_dtype, (int)T, vec, grid, g_spikes, g_vfinal, x, spikes, beta, v_th,
                                    v_reset, in_gain, surrogate_kind, surrogate_k, c, grad_x, partials, N, st);
      break;
    default: return fail(SPK_ERR_INVALID, "x dtype %d not supported", x_dtype);
  }
  if (rc != SPK_OK) return rc;
  if ((rc = check_launch("lif_bwd_kernel")) != SPK_OK) return rc;
  if (grad_beta) {
    sum_partials_kernel<<<1, 1024, 0, st>>>(partials, grid, grad_beta);
    if ((rc = check_launch("sum_partials_kernel")) != SPK_OK) return rc;
  }
  return SPK_OK;
}

static int check_lif_args(const void* x, int x_dtype, const void* spikes, int spike_dtype, const float* beta,
                          const float* v_th, const float* v_reset, int64_t T, int64_t N) {
  // an empty tensor may carry a null data pointer
  SPK_REQUIRE((x && spikes) || N == 0, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(beta && v_th && v_reset, SPK_ERR_INVALID, "null pointer argument");
  SPK_REQUIRE(x_dtype == SPK_F32 || x_dtype == SPK_F16 || x_dtype == SPK_BF16, SPK_ERR_INVALID,
              "x dtype %d not supported", x_dtype);
  SPK_REQUIRE(spike_dtype == SPK_F32 || spike_dtype == SPK_BF16 || spike_dtype == SPK_U8 ||
                  spike_dtype == SPK_FP8 || spike_dtype == SPK_BIT,
              SPK_ERR_INVALID, "spike dtype %d not supported", spike_dtype);
  SPK_REQUIRE(T >= 1 && T <= 64, SPK_ERR_SHAPE, "T=%lld outside [1, 64]", (long long)T);
  SPK_REQUIRE(N >= 0, SPK_ERR_SHAPE, "N=%lld negative", (long long)N);
  SPK_REQUIRE(aligned(x, dtype_size(x_dtype)) && (spike_dtype == SPK_BIT || aligned(spikes, dtype_size(spike_dtype))),
              SPK_ERR_ALIGN, "x / spikes not aligned to their element size");
  return SPK_OK;
}

// ---- allocation-free backward (spk_lif_bwd_noalloc) ----------------------
// Some callers cannot allocate device memory: code that runs while a custom
// caching allocator owns the whole device heap, plugin hosts whose memory
// budget is fixed up front, or callers without a device allocator of their
// own (plain C, FFI).  For them the grad_beta partial sums live in this
// file-scope array instead of a caller-provided workspace.  It holds
// kNoAllocScratchFloats = 4096 floats (16 KiB), the largest grid the backward
// kernel ever launches (kBwdMaxBlocks), so no N is too large for it; a call
// whose grid would need more partial sums is rejected with SPK_ERR_SHAPE.
// Every call on a device shares the array and it keeps the last call's
// contents.  Nothing in it has to start at zero: each block writes its own
// partial before the reduction kernel, stream-ordered after it, reads
// partials [0, grid).  Calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array.
constexpr int kNoAllocScratchFloats = 4096;
static_assert(kNoAllocScratchFloats >= kBwdMaxBlocks, "scratch must cover the largest backward grid");
static __device__ __align__(256) float g_lif_bwd_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;

// Device address of g_lif_bwd_scratch on the current device.  The first call
// on a device resolves it with cudaGetSymbolAddress (with that device
// current, which loads the module there if it is not loaded yet); later calls
// reuse the cached address.
static int noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[kNoAllocMaxDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  SPK_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, SPK_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev,
              kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lif_bwd_scratch);
    if (e != cudaSuccess || !p)
      return fail(SPK_ERR_CUDA, "cudaGetSymbolAddress(LIF backward scratch) on device %d: %s", dev,
                  cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return SPK_OK;
}

// Upper bound on the grid lif_bwd_impl launches for (T, N): the scalar path
// (one neuron per thread) gives the larger grid, and both are capped at
// kBwdMaxBlocks.
static int64_t noalloc_partials_needed(int64_t N) {
  int64_t g = grid_for(N, kBwdThreads);
  return g > kBwdMaxBlocks ? kBwdMaxBlocks : g;
}

}  // namespace spk

extern "C" {

int spk_lif_fwd(const void* x, int x_dtype, void* spikes, int spike_dtype, float* v_final, const float* beta,
                const float* v_th, const float* v_reset, float in_gain, int64_t T, int64_t N, void* stream) {
  using namespace spk;
  int rc = check_lif_args(x, x_dtype, spikes, spike_dtype, beta, v_th, v_reset, T, N);
  if (rc != SPK_OK) return rc;
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  if (N == 0) return SPK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = (N % 8 == 0) && aligned(x, 8 * dtype_size(x_dtype)) &&
                   (spike_dtype == SPK_BIT || aligned(spikes, 8 * dtype_size(spike_dtype))) &&
                   (!v_final || aligned(v_final, 32));
  switch (x_dtype) {
    case SPK_F32: rc = dispatch_fwd_s<SPK_F32>(spike_dtype, vec, x, spikes, v_final, beta, v_th, v_reset, in_gain, (int)T, N, st); break;
    case SPK_F16: rc = dispatch_fwd_s<SPK_F16>(spike_dtype, vec, x, spikes, v_final, beta, v_th, v_reset, in_gain, (int)T, N, st); break;
    default: rc = dispatch_fwd_s<SPK_BF16>(spike_dtype, vec, x, spikes, v_final, beta, v_th, v_reset, in_gain, (int)T, N, st); break;
  }
  if (rc != SPK_OK) return rc;
  return check_launch("lif_fwd_kernel");
}

int64_t spk_lif_bwd_workspace_bytes(int64_t T, int64_t N) {
  (void)T;
  (void)N;
  return (int64_t)spk::kBwdMaxBlocks * (int64_t)sizeof(float);
}

int spk_lif_bwd(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype, const void* spikes,
                int spike_dtype, const float* beta, const float* v_th, const float* v_reset, float in_gain,
                int surrogate, float surrogate_k, void* grad_x, float* grad_beta, void* workspace,
                int64_t workspace_bytes, int64_t T, int64_t N, void* stream) {
  using namespace spk;
  int rc = check_lif_args(x, x_dtype, spikes, spike_dtype, beta, v_th, v_reset, T, N);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE((g_spikes && grad_x) || N == 0, SPK_ERR_INVALID, "null gradient pointer");
  SPK_REQUIRE(surrogate == SPK_SURROGATE_SUPERSPIKE || surrogate == SPK_SURROGATE_ARCTAN, SPK_ERR_INVALID,
              "unknown surrogate %d", surrogate);
  SPK_REQUIRE(aligned(g_spikes, 4) && aligned(grad_x, dtype_size(x_dtype)), SPK_ERR_ALIGN,
              "gradient pointers misaligned");
  if (grad_beta) {
    SPK_REQUIRE(workspace && workspace_bytes >= spk_lif_bwd_workspace_bytes(T, N), SPK_ERR_INVALID,
                "workspace of %lld bytes is smaller than spk_lif_bwd_workspace_bytes() = %lld",
                (long long)workspace_bytes, (long long)spk_lif_bwd_workspace_bytes(T, N));
    SPK_REQUIRE(aligned(workspace, 4), SPK_ERR_ALIGN, "workspace misaligned");
  }
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (N == 0) {
    if (grad_beta) cudaMemsetAsync(grad_beta, 0, sizeof(float), st);
    return SPK_OK;
  }
  return lif_bwd_impl(g_spikes, g_vfinal, x, x_dtype, spikes, spike_dtype, beta, v_th, v_reset, in_gain,
                      surrogate, surrogate_k, grad_x, grad_beta, reinterpret_cast<float*>(workspace), T, N, st);
}

int spk_lif_bwd_noalloc(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype,
                        const void* spikes, int spike_dtype, const float* beta, const float* v_th,
                        const float* v_reset, float in_gain, int surrogate, float surrogate_k, void* grad_x,
                        float* grad_beta, int64_t T, int64_t N, void* stream) {
  using namespace spk;
  int rc = check_lif_args(x, x_dtype, spikes, spike_dtype, beta, v_th, v_reset, T, N);
  if (rc != SPK_OK) return rc;
  SPK_REQUIRE((g_spikes && grad_x) || N == 0, SPK_ERR_INVALID, "null gradient pointer");
  SPK_REQUIRE(surrogate == SPK_SURROGATE_SUPERSPIKE || surrogate == SPK_SURROGATE_ARCTAN, SPK_ERR_INVALID,
              "unknown surrogate %d", surrogate);
  SPK_REQUIRE(aligned(g_spikes, 4) && aligned(grad_x, dtype_size(x_dtype)), SPK_ERR_ALIGN,
              "gradient pointers misaligned");
  if ((rc = check_stream_device(stream)) != SPK_OK) return rc;
  const int64_t need = noalloc_partials_needed(N);
  SPK_REQUIRE(need <= kNoAllocScratchFloats, SPK_ERR_SHAPE,
              "N=%lld needs %lld grad_beta partial sums; the static scratch holds %d", (long long)N,
              (long long)need, kNoAllocScratchFloats);
  float* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch)) != SPK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (N == 0) {
    if (grad_beta) {
      cudaError_t e = cudaMemsetAsync(grad_beta, 0, sizeof(float), st);
      if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
    return SPK_OK;
  }
  return lif_bwd_impl(g_spikes, g_vfinal, x, x_dtype, spikes, spike_dtype, beta, v_th, v_reset, in_gain,
                      surrogate, surrogate_k, grad_x, grad_beta, scratch, T, N, st);
}

}  // extern "C"
