// CNN policy trunk (train/model.py:77-101, 187-190): conv0 3x3 (14->16, the
// seat's view permutation folded into its input-channel order) -> LN[16,H,W]
// -> ReLU -> conv 3x3 16->32 -> LN -> ReLU -> conv 3x3 32->64 -> LN -> ReLU
// -> conv 1x1 64->8 -> LN -> ReLU -> flatten -> Linear(8HW -> 128).
// The output (first Linear incl. bias) goes to the same pre-activation buffer
// as the MLP's first layer; k_mlp_heads then runs the shared tail
// (LN, ReLU, 128x128, LN, ReLU, heads, masking, sampling) unchanged, because
// the CNN's `shared` stack after its first Linear is the MLP's.
//
// One block (256 threads) per (env, seat).  Activations live in shared
// memory as zero-bordered (H+2)x(W+2) planes; a work item is 4 output
// channels of one pixel; the LayerNorms are block reductions.  fp32 FMA on
// the CUDA cores (first version; a tensor-core implicit GEMM is the next
// step).

#include "qqt_common.cuh"

namespace qqt {

constexpr int kCnnThreads = 256;

struct CnnPackLayout {
  // float offsets
  size_t w0, b0, g0, be0, w1, b1, g1, be1, w2, b2, g2, be2, w3, b3, g3, be3, wl, bl, tail, total;
};

__host__ __device__ inline CnnPackLayout cnn_layout(int c_in, int hw, int n_seats) {
  CnnPackLayout L;
  size_t o = 0;
  auto take = [&](size_t n) {
    const size_t at = o;
    o += (n + 63) & ~(size_t)63;
    return at;
  };
  L.w0 = take((size_t)n_seats * 16 * c_in * 9);
  L.b0 = take(16);
  L.g0 = take((size_t)16 * hw);
  L.be0 = take((size_t)16 * hw);
  L.w1 = take(32 * 16 * 9);
  L.b1 = take(32);
  L.g1 = take((size_t)32 * hw);
  L.be1 = take((size_t)32 * hw);
  L.w2 = take(64 * 32 * 9);
  L.b2 = take(64);
  L.g2 = take((size_t)64 * hw);
  L.be2 = take((size_t)64 * hw);
  L.w3 = take(8 * 64);
  L.b3 = take(8);
  L.g3 = take((size_t)8 * hw);
  L.be3 = take((size_t)8 * hw);
  L.wl = take((size_t)8 * hw * 128);   // transposed [8*hw][128]
  L.bl = take(128);
  L.tail = take(F_TOTAL);
  L.total = o;
  return L;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = __fadd_rn(v, 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(QQT_FULL, v, o);
  __syncthreads();
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kCnnThreads / 32; ++i) s += red[i];
  return s;
}

// out[oc][interior] = bias[oc] + sum_ic sum_taps w[oc][ic][tap] * in[ic][...]
template <int CIN, int COUT, int KS>
__device__ __forceinline__ void conv_layer(const float* in, float* out, const float* __restrict__ w,
                                           const float* __restrict__ b, int h, int wd) {
  const int pw = wd + 2, pp = (h + 2) * pw, hw = h * wd;
  const int items = (COUT / 4) * hw;
  for (int it = threadIdx.x; it < items; it += kCnnThreads) {
    const int og = it / hw, p = it - og * hw;
    const int r = p / wd, c = p - r * wd;
    float acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = __ldg(b + 4 * og + j);
    const float* wb = w + (size_t)(4 * og) * CIN * KS * KS;
    for (int ic = 0; ic < CIN; ++ic) {
      const float* ip = in + ic * pp + (r + 1 - KS / 2) * pw + (c + 1 - KS / 2);
#pragma unroll
      for (int ky = 0; ky < KS; ++ky)
#pragma unroll
        for (int kx = 0; kx < KS; ++kx) {
          const float x = ip[ky * pw + kx];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[j] = fmaf(__ldg(wb + ((size_t)j * CIN + ic) * KS * KS + ky * KS + kx), x, acc[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out[(4 * og + j) * pp + (r + 1) * pw + (c + 1)] = acc[j];
  }
  __syncthreads();
}

// LayerNorm over all C*h*w interior values with elementwise affine, then ReLU.
__device__ __forceinline__ void ln_relu_map(float* buf, int C, const float* __restrict__ g,
                                            const float* __restrict__ be, int h, int wd,
                                            float* red) {
  const int pw = wd + 2, pp = (h + 2) * pw, hw = h * wd, n = C * hw;
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += kCnnThreads) {
    const int c = i / hw, p = i - c * hw, r = p / wd, q = p - r * wd;
    s += buf[c * pp + (r + 1) * pw + q + 1];
  }
  const float mean = block_sum(s, red) / (float)n;
  float v = 0.f;
  for (int i = threadIdx.x; i < n; i += kCnnThreads) {
    const int c = i / hw, p = i - c * hw, r = p / wd, q = p - r * wd;
    const float d = buf[c * pp + (r + 1) * pw + q + 1] - mean;
    v = fmaf(d, d, v);
  }
  const float rstd = rsqrtf(block_sum(v, red) / (float)n + 1e-5f);
  for (int i = threadIdx.x; i < n; i += kCnnThreads) {
    const int c = i / hw, p = i - c * hw, r = p / wd, q = p - r * wd;
    float* x = buf + c * pp + (r + 1) * pw + q + 1;
    *x = fmaxf(fmaf((*x - mean) * rstd, __ldg(g + i), __ldg(be + i)), 0.f);
  }
  __syncthreads();
}

template <int CIN0>
__global__ void __launch_bounds__(kCnnThreads)
k_cnn_trunk(const __half* __restrict__ obs, int obs_stride, int n, const float* __restrict__ pk,
            int n_seats, int h, int wd, float* __restrict__ pre) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[kCnnThreads / 32];
  const int e = blockIdx.x, seat = blockIdx.y;
  const int pw = wd + 2, pp = (h + 2) * pw, hw = h * wd;
  const CnnPackLayout L = cnn_layout(CIN0, hw, n_seats);
  float* A = sm;                 // up to 32 planes
  float* B = sm + 32 * pp;       // up to 64 planes
  for (int i = threadIdx.x; i < 96 * pp; i += kCnnThreads) sm[i] = 0.f;
  __syncthreads();
  const __half* orow = obs + (size_t)e * obs_stride;
  for (int i = threadIdx.x; i < CIN0 * hw; i += kCnnThreads) {
    const int c = i / hw, p = i - c * hw, r = p / wd, q = p - r * wd;
    A[c * pp + (r + 1) * pw + q + 1] = __half2float(orow[i]);
  }
  __syncthreads();
  conv_layer<CIN0, 16, 3>(A, B, pk + L.w0 + (size_t)seat * 16 * CIN0 * 9, pk + L.b0, h, wd);
  ln_relu_map(B, 16, pk + L.g0, pk + L.be0, h, wd, red);
  // the conv outputs only ever write interiors: borders stay zero
  conv_layer<16, 32, 3>(B, A, pk + L.w1, pk + L.b1, h, wd);
  ln_relu_map(A, 32, pk + L.g1, pk + L.be1, h, wd, red);
  conv_layer<32, 64, 3>(A, B, pk + L.w2, pk + L.b2, h, wd);
  ln_relu_map(B, 64, pk + L.g2, pk + L.be2, h, wd, red);
  conv_layer<64, 8, 1>(B, A, pk + L.w3, pk + L.b3, h, wd);
  ln_relu_map(A, 8, pk + L.g3, pk + L.be3, h, wd, red);
  // flatten (channel-major) -> Linear(8*hw -> 128): two threads per output
  float* flat = B;               // compact copy of the 8 planes
  for (int i = threadIdx.x; i < 8 * hw; i += kCnnThreads) {
    const int c = i / hw, p = i - c * hw, r = p / wd, q = p - r * wd;
    flat[i] = A[c * pp + (r + 1) * pw + q + 1];
  }
  __syncthreads();
  const int o = threadIdx.x & 127, half = threadIdx.x >> 7;
  const int k_in = 8 * hw, k0 = half * (k_in / 2), k1 = half ? k_in : k_in / 2;
  float acc = 0.f;
  const float* wl = pk + L.wl;
  for (int k = k0; k < k1; ++k) acc = fmaf(__ldg(wl + (size_t)k * 128 + o), flat[k], acc);
  float* part = flat + k_in;
  if (half) part[o] = acc;
  __syncthreads();
  if (!half) pre[(size_t)e * (128 * n_seats) + seat * 128 + o] = acc + part[o] + __ldg(pk + L.bl + o);
}

struct CnnParams {
  const float* p[18];   // conv stack + shared.0 (see qqt_cnn_param_names)
};

__global__ void k_cnn_pack(CnnParams prm, int c_in, int hw, int n_seats, SeatChannels sc,
                           float* __restrict__ pk) {
  const CnnPackLayout L = cnn_layout(c_in, hw, n_seats);
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  // conv0 with the seat's input-channel gather: stored channel k reads W0[:, inv[k]]
  if (i < (size_t)n_seats * 16 * c_in * 9) {
    const int s = (int)(i / (16 * c_in * 9));
    const int rem = (int)(i % (16 * c_in * 9));
    const int oc = rem / (c_in * 9), k = (rem / 9) % c_in, tap = rem % 9;
    pk[L.w0 + i] = prm.p[0][((size_t)oc * c_in + sc.src[s][k]) * 9 + tap];
  }
  if (i < 16) pk[L.b0 + i] = prm.p[1][i];
  if (i < (size_t)16 * hw) { pk[L.g0 + i] = prm.p[2][i]; pk[L.be0 + i] = prm.p[3][i]; }
  if (i < 32 * 16 * 9) pk[L.w1 + i] = prm.p[4][i];
  if (i < 32) pk[L.b1 + i] = prm.p[5][i];
  if (i < (size_t)32 * hw) { pk[L.g1 + i] = prm.p[6][i]; pk[L.be1 + i] = prm.p[7][i]; }
  if (i < 64 * 32 * 9) pk[L.w2 + i] = prm.p[8][i];
  if (i < 64) pk[L.b2 + i] = prm.p[9][i];
  if (i < (size_t)64 * hw) { pk[L.g2 + i] = prm.p[10][i]; pk[L.be2 + i] = prm.p[11][i]; }
  if (i < 8 * 64) pk[L.w3 + i] = prm.p[12][i];
  if (i < 8) pk[L.b3 + i] = prm.p[13][i];
  if (i < (size_t)8 * hw) { pk[L.g3 + i] = prm.p[14][i]; pk[L.be3 + i] = prm.p[15][i]; }
  if (i < (size_t)128 * 8 * hw) {
    const int o = (int)(i / (8 * hw)), k = (int)(i % (8 * hw));   // shared.0.weight [128][8hw]
    pk[L.wl + (size_t)k * 128 + o] = prm.p[16][i];
  }
  if (i < 128) pk[L.bl + i] = prm.p[17][i];
}

}  // namespace qqt

using namespace qqt;

static const char* kCnnNames =
    "conv0.weight conv0.bias conv.0.weight conv.0.bias conv.2.weight conv.2.bias conv.3.weight "
    "conv.3.bias conv.5.weight conv.5.bias conv.6.weight conv.6.bias conv.8.weight conv.8.bias "
    "conv.9.weight conv.9.bias shared.0.weight shared.0.bias shared.1.weight shared.1.bias "
    "shared.3.weight shared.3.bias shared.4.weight shared.4.bias move_head.0.weight "
    "move_head.0.bias move_head.2.weight move_head.2.bias bomb_head.0.weight bomb_head.0.bias "
    "bomb_head.2.weight bomb_head.2.bias critic.0.weight critic.0.bias critic.2.weight "
    "critic.2.bias";

extern "C" const char* qqt_cnn_param_names(void) { return kCnnNames; }

extern "C" uint64_t qqt_cnn_pack_bytes(int32_t channels, int32_t hw, int32_t n_seats) {
  if (channels != 14 || hw <= 0 || n_seats < 1 || n_seats > 2) return 0;
  return cnn_layout(channels, hw, n_seats).total * 4;
}

extern "C" int qqt_cnn_pack(const float* const* params_dev, int32_t n_players, int32_t channels,
                            int32_t hw, int32_t n_seats, const int32_t* pids, void* pack,
                            qqt_stream_t stream) {
  if (!params_dev || !pack || !pids || channels != 14 || n_seats < 1 || n_seats > 2)
    return QQT_E_ARG;
  if (n_players < 2 || n_players > QQT_MAX_P) return QQT_E_ARG;
  SeatChannels sc;
  memset(&sc, 0, sizeof(sc));
  const int base = 2 * n_players + 3;
  for (int s = 0; s < n_seats; ++s) {
    const int me = pids[s];
    if (me < 0 || me >= n_players) return QQT_E_ARG;
    int perm[64], j = 0;
    perm[j++] = me;
    perm[j++] = n_players + me;
    for (int i = 0; i < n_players; ++i)
      if (i != me) perm[j++] = i;
    for (int i = 0; i < n_players; ++i)
      if (i != me) perm[j++] = n_players + i;
    perm[j++] = 2 * n_players;
    perm[j++] = 2 * n_players + 1;
    perm[j++] = 2 * n_players + 2;
    for (int c = base; c < channels; ++c) perm[j++] = c;
    for (int v = 0; v < channels; ++v) sc.src[s][perm[v]] = v;
  }
  for (int i = 0; i < 36; ++i)
    if (!params_dev[i]) return QQT_E_ARG;
  const CnnPackLayout L = cnn_layout(channels, hw, n_seats);
  float* pk = (float*)pack;
  cudaStream_t st = (cudaStream_t)stream;
  CnnParams cp;
  for (int i = 0; i < 18; ++i) cp.p[i] = params_dev[i];
  const size_t n_items = (size_t)128 * 8 * hw;
  k_cnn_pack<<<(unsigned)((n_items + 255) / 256), 256, 0, st>>>(cp, channels, hw, n_seats, sc, pk);
  // shared tail (LN, 128x128, LN, heads) in the MLP pack's float layout
  HeadParams hp;
  // q[] uses the MLP's parameter order: q[0] = shared.0.weight (index 16),
  // q[1] = shared.0.bias, q[2] = shared.1.weight, ..., q[19] = critic.2.bias (35)
  const float* const* q = params_dev + 16;
  hp.b0 = q[1];
  hp.ln1g = q[2];
  hp.ln1b = q[3];
  hp.w1 = q[4];
  hp.b1 = q[5];
  hp.ln2g = q[6];
  hp.ln2b = q[7];
  hp.mw0 = q[8];
  hp.mb0 = q[9];
  hp.mw2 = q[10];
  hp.mb2 = q[11];
  hp.bw0 = q[12];
  hp.bb0 = q[13];
  hp.bw2 = q[14];
  hp.bb2 = q[15];
  hp.cw0 = q[16];
  hp.cb0 = q[17];
  hp.cw2 = q[18];
  hp.cb2 = q[19];
  k_mlp_pack_rest<<<(128 * 128 + 255) / 256, 256, 0, st>>>(hp, n_seats, pk + L.tail);
  return launch_status();
}

extern "C" uint64_t qqt_cnn_work_bytes(int32_t n_envs, int32_t n_seats) {
  return (uint64_t)n_envs * 128 * n_seats * 4;
}

extern "C" int qqt_cnn_act(const void* pack, const void* obs, int32_t n_envs, int32_t obs_stride,
                           int32_t height, int32_t width, int32_t channels, int32_t n_seats,
                           const uint8_t* const* mm, int32_t mm_stride, const uint8_t* const* bm,
                           int32_t bm_stride, const float* u, int64_t* const* act,
                           int32_t act_stride, float* logp, float* value, float* logits,
                           void* work, qqt_stream_t stream) {
  if (!pack || !obs || !mm || !bm || !u || !act || !work || channels != 14) return QQT_E_ARG;
  if (n_envs <= 0 || n_seats < 1 || n_seats > 2 || height > QQT_MAX_H || width > QQT_MAX_W ||
      mm_stride < 5 || bm_stride < 2 || act_stride < 2)
    return QQT_E_ARG;
  if (obs_stride < channels * height * width) return QQT_E_ALIGN;
  for (int s = 0; s < n_seats; ++s)
    if (!mm[s] || !bm[s] || !act[s]) return QQT_E_ARG;
  const int hw = height * width;
  const CnnPackLayout L = cnn_layout(channels, hw, n_seats);
  const float* pk = (const float*)pack;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t sm = (size_t)96 * (height + 2) * (width + 2) * 4;
  cudaFuncSetAttribute(k_cnn_trunk<14>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  float* pre = (float*)work;
  k_cnn_trunk<14><<<dim3(n_envs, n_seats), kCnnThreads, sm, st>>>(
      (const __half*)obs, obs_stride, n_envs, pk, n_seats, height, width, pre);
  for (int s = 0; s < n_seats; ++s)
    k_mlp_heads<<<(n_envs + kHR - 1) / kHR, 128, 0, st>>>(pre, 128 * n_seats, s, n_envs,
                                                           pk + L.tail, mm[s], mm_stride, bm[s],
                                                           bm_stride, u, act[s], act_stride, logp,
                                                           value, logits);
  return launch_status();
}
