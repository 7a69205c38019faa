// CNN policy (train/model.py:77-101, 187-196) on the 5th-generation tensor
// cores.
//
// Trunk: conv0 3x3 (14 -> 16, the seat's view permutation folded into its
// input-channel order) -> LN[16,H,W] -> ReLU -> conv 3x3 16 -> 32 -> LN ->
// ReLU -> conv 3x3 32 -> 64 -> LN -> ReLU -> conv 1x1 64 -> 8 -> LN -> ReLU
// -> flatten (c*HW + y*W + x).
//
// k_cnn_trunk (persistent, one CTA of 8 warps per SM, one sample at a
// time): the sample's activation lives in shared memory as a zero-bordered
// 15x15 pixel grid, one 128-byte row per pixel (channels K-major, fp16 hi
// and lo halves, 128-byte swizzle) with 16 margin rows on each side.  A 3x3
// convolution is then nine GEMMs whose A operands are the same buffer
// shifted by (ky-1)*15 + (kx-1) rows: the descriptor's start address moves,
// nothing is copied (the swizzle follows absolute shared-memory address
// bits, so any row offset is a valid operand start).  Each layer runs
// M = 2 x 128 padded pixels (225 used, border rows ignored), K = Cin per
// tap.  The weights' fp16 hi and lo halves are stacked along N, so one MMA
// A_hi * [W_hi; W_lo] (N = 2 Cout) gives the hi*hi and hi*lo products in two
// column halves and a second A_lo * W_hi (N = Cout) accumulates into the
// first half (conv0's input is the exact fp16 observation: one MMA); the
// epilogue adds the halves.  All conv weights stay resident in shared
// memory as pre-swizzled images (one bulk copy per CTA).  The epilogue (thread = TMEM lane = pixel
// row, two warps per lane quadrant splitting the channels) adds the bias,
// computes the sample's LayerNorm statistics with two block reductions (mean, then the centred sum of squares), applies the
// affine LN and ReLU, splits into fp16 hi/lo and writes the next layer's
// input into the same buffer; the last layer writes the flattened
// activation to global memory as fp16 hi and lo rows of 1408 (1352 + zero
// pad).
//
// Linear(1352 -> 128) and the shared tail (LN, ReLU, 128x128, LN, ReLU,
// heads, masking, sampling) are k_mlp_fused with a split A operand.
//
// Geometry: H = W = 13 (the reference's board), P = 2 channel layout (C=14).

#include "qqt_common.cuh"

namespace qqt {

constexpr int kCnnH = 13, kCnnW = 13, kCnnHW = 169, kCnnPW = 15, kCnnPP = 225;
constexpr int kCnnKIn = 8 * kCnnHW;                  // 1352 flattened features
constexpr int kCnnKP = 1408;                         // padded to 22 K tiles of 64
constexpr int kActMargin = 16, kActRows = 288;       // 16 + 256 + 16
constexpr int kActBytes = kActRows * 128;            // one of hi / lo
// weight images (bytes): per group of taps, 2 x Cout rows of 128 bytes (hi
// rows, then lo rows); conv0 3 groups (4 taps of 16 channels per row),
// conv1 3 groups, conv2 5 groups (2 taps of 32), conv3 1 group (Cout padded
// to 16)
constexpr int kW0 = 3 * 32 * 128, kW1 = 3 * 64 * 128, kW2 = 5 * 128 * 128, kW3 = 32 * 128;

struct CnnLayout {
  size_t c0, c1, c2, c3, wbytes;          // image offsets (bytes); c0 is per seat
  size_t lnf;                             // float block (bytes offset)
  size_t mlp, total;                      // embedded MLP pack of the linear + tail
};
// float block (floats from lnf): LN gamma/beta [HW][C] per layer, conv biases
enum {
  LF_G0 = 0, LF_B0 = LF_G0 + 16 * kCnnHW, LF_G1 = LF_B0 + 16 * kCnnHW,
  LF_B1 = LF_G1 + 32 * kCnnHW, LF_G2 = LF_B1 + 32 * kCnnHW, LF_B2 = LF_G2 + 64 * kCnnHW,
  LF_G3 = LF_B2 + 64 * kCnnHW, LF_B3 = LF_G3 + 8 * kCnnHW, LF_CB0 = LF_B3 + 8 * kCnnHW,
  LF_CB1 = LF_CB0 + 16, LF_CB2 = LF_CB1 + 32, LF_CB3 = LF_CB2 + 64, LF_TOTAL = LF_CB3 + 8
};

__host__ __device__ inline CnnLayout cnn_layout(int n_seats) {
  CnnLayout L;
  L.c0 = 0;
  L.c1 = (size_t)n_seats * kW0;
  L.c2 = L.c1 + kW1;
  L.c3 = L.c2 + kW2;
  L.wbytes = L.c3 + kW3;
  L.lnf = (L.wbytes + 255) / 256 * 256;
  L.mlp = (L.lnf + (size_t)LF_TOTAL * 4 + 1023) / 1024 * 1024;
  L.total = L.mlp + mlp_pack_layout(kCnnKIn, 1).total;
  return L;
}

// ------------------------------------------------------------ pack

struct CnnParams {
  const float* p[16];   // conv stack (qqt_cnn_param_names order)
};

// Weight (n, k) of a group image with C output rows: hi at row n, lo at
// row C + n (128-byte swizzled K-major rows).
__device__ __forceinline__ void put_split(uint8_t* group, int C, int n, int k, float v) {
  const __half hi = __float2half_rn(v);
  const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
  *reinterpret_cast<__half*>(group + sw128_off(n, k, 2 * C)) = hi;
  *reinterpret_cast<__half*>(group + sw128_off(C + n, k, 2 * C)) = lo;
}

// Conv weights -> swizzled hi/lo images; LN affine and conv biases -> floats.
__global__ void k_cnn_pack(CnnParams prm, int n_seats, SeatChannels sc, uint8_t* __restrict__ pk) {
  const CnnLayout L = cnn_layout(n_seats);
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  // conv0: (seat, group, n, k) -> tap g*4 + k/16, stored channel k%16
  if (i < n_seats * 3 * 16 * 64) {
    const int s = i / (3 * 16 * 64), r = i % (3 * 16 * 64);
    const int g = r / (16 * 64), n = (r / 64) % 16, k = r % 64;
    const int t = g * 4 + k / 16, ic = k % 16;
    const float v = (t < 9 && ic < 14) ? prm.p[0][((size_t)n * 14 + sc.src[s][ic]) * 9 + t] : 0.f;
    put_split(pk + L.c0 + (size_t)s * kW0 + g * 32 * 128, 16, n, k, v);
  }
  if (i < 3 * 32 * 64) {
    const int g = i / (32 * 64), n = (i / 64) % 32, k = i % 64;
    const int t = g * 4 + k / 16, ic = k % 16;
    const float v = t < 9 ? prm.p[4][((size_t)n * 16 + ic) * 9 + t] : 0.f;
    put_split(pk + L.c1 + g * 64 * 128, 32, n, k, v);
  }
  if (i < 5 * 64 * 64) {
    const int g = i / (64 * 64), n = (i / 64) % 64, k = i % 64;
    const int t = g * 2 + k / 32, ic = k % 32;
    const float v = t < 9 ? prm.p[8][((size_t)n * 32 + ic) * 9 + t] : 0.f;
    put_split(pk + L.c2 + g * 128 * 128, 64, n, k, v);
  }
  if (i < 16 * 64) {
    const int n = i / 64, k = i % 64;
    const float v = n < 8 ? prm.p[12][(size_t)n * 64 + k] : 0.f;
    put_split(pk + L.c3, 16, n, k, v);
  }
  // LN affine [C][H][W] -> [pixel][C] (a pixel's channels contiguous)
  float* f = (float*)(pk + L.lnf);
  auto tr = [&](int C, int off_g, int off_b, const float* g, const float* b) {
    if (i < C * kCnnHW) {
      const int c = i / kCnnHW, px = i % kCnnHW;
      f[off_g + px * C + c] = g[i];
      f[off_b + px * C + c] = b[i];
    }
  };
  tr(16, LF_G0, LF_B0, prm.p[2], prm.p[3]);
  tr(32, LF_G1, LF_B1, prm.p[6], prm.p[7]);
  tr(64, LF_G2, LF_B2, prm.p[10], prm.p[11]);
  tr(8, LF_G3, LF_B3, prm.p[14], prm.p[15]);
  if (i < 16) f[LF_CB0 + i] = prm.p[1][i];
  if (i < 32) f[LF_CB1 + i] = prm.p[5][i];
  if (i < 64) f[LF_CB2 + i] = prm.p[9][i];
  if (i < 8) f[LF_CB3 + i] = prm.p[13][i];
}

// ------------------------------------------------------------ trunk

// tcgen05.ld of NC (4, 8 or 16) consecutive 32-bit columns of this lane.
template <int NC>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, float* v) {
  uint32_t r[16];
  if (NC == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  } else if (NC == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < NC; ++i) v[i] = __uint_as_float(r[i]);
}

constexpr int kTrunkWarps = 8;    // 2 per TMEM lane quadrant, splitting the columns

// Sum over the CTA's threads (every thread gets the total; fixed order).
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(QQT_FULL, v, o);
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kTrunkWarps; ++i) s += red[i];
  __syncthreads();
  return s;
}

// Padded-grid row r (0..255) -> interior pixel index, or -1.
__device__ __forceinline__ int interior_pixel(int r) {
  if (r >= kCnnPP) return -1;
  const int py = r / kCnnPW, px = r - py * kCnnPW;
  if (py < 1 || py > kCnnH || px < 1 || px > kCnnW) return -1;
  return (py - 1) * kCnnW + (px - 1);
}

// One conv layer's MMAs: two M tiles of 128 padded rows (TMEM columns
// [128 j, 128 j + 2C)), `taps` taps (3x3: the A operand of tap (ky,kx) starts
// (ky-1)*15 + (kx-1) rows away), CIN/16 K steps per tap; tap t's weights sit
// in group t / (64 / CIN) at byte (t % (64 / CIN)) * CIN * 2 of each row.
template <int C, int CIN, int TAPS, bool SPLIT>
__device__ __forceinline__ void conv_mma(uint32_t tmem, const uint8_t* act_hi, const uint8_t* act_lo,
                                         const uint8_t* w) {
  constexpr int TPG = 64 / CIN;
  const uint32_t id2 = idesc_f16(128, 2 * C), id1 = idesc_f16(128, C);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint32_t d = tmem + 128 * j;
#pragma unroll
    for (int t = 0; t < TAPS; ++t) {
      const int shift = TAPS == 9 ? (t / 3 - 1) * kCnnPW + (t % 3 - 1) : 0;
      const int arow = kActMargin + j * 128 + shift;
      const uint32_t wb = (t / TPG) * 2 * C * 128 + (t % TPG) * CIN * 2;
      const uint64_t ah = sw128_desc(act_hi + arow * 128), al = sw128_desc(act_lo + arow * 128);
      const uint64_t bw = sw128_desc(w + wb);
#pragma unroll
      for (int kk = 0; kk < CIN / 16; ++kk) {
        const uint64_t o = (uint64_t)(kk * 2);       // 32 bytes per K = 16 step
        umma_f16(d, ah + o, bw + o, id2, (t > 0 || kk > 0) ? 1u : 0u);
        if (SPLIT) umma_f16(d, al + o, bw + o, id1, 1u);
      }
    }
  }
}

// Epilogue of one layer.  Warp w reads TMEM lane quadrant w % 4 (padded
// rows q*32 + lane of both M tiles) and column half w / 4 (NC = N / 2
// channels); bias, the sample's LayerNorm over NREAL x HW values, ReLU.
// The LN affine parameters of the thread's two pixels are loaded as 16-byte
// vectors ([pixel][C] layout) before the statistics are reduced.
// !FINAL: the result goes back into the activation buffer as the next
// layer's fp16 hi/lo input; FINAL: flattened (c * HW + pixel) into the
// global hi / lo rows.
// The LN affine parameters of the thread's two pixels ([pixel][C] layout,
// 16-byte loads; the caller issues this before waiting for the layer's MMAs,
// so the loads overlap them).
template <int N, int NREAL>
__device__ __forceinline__ void ln_params(const float* __restrict__ lnf, int lg, int lb, float* g0,
                                          float* b0, float* g1, float* b1) {
  constexpr int NC = N / 2;
  const int w = warp_id(), q = w & 3, cg = w >> 2, lane = lane_id();
  const int c0 = cg * NC;
  const bool real = c0 < NREAL;
  const int r0 = q * 32 + lane, r1 = 128 + r0;
  const int p0 = real ? interior_pixel(r0) : -1, p1 = real ? interior_pixel(r1) : -1;
#pragma unroll
  for (int c = 0; c < NC; c += 4) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 ga = p0 >= 0 ? __ldg(reinterpret_cast<const float4*>(lnf + lg + p0 * NREAL + c0 + c)) : z;
    const float4 ba = p0 >= 0 ? __ldg(reinterpret_cast<const float4*>(lnf + lb + p0 * NREAL + c0 + c)) : z;
    const float4 gb = p1 >= 0 ? __ldg(reinterpret_cast<const float4*>(lnf + lg + p1 * NREAL + c0 + c)) : z;
    const float4 bb = p1 >= 0 ? __ldg(reinterpret_cast<const float4*>(lnf + lb + p1 * NREAL + c0 + c)) : z;
    g0[c] = ga.x; g0[c + 1] = ga.y; g0[c + 2] = ga.z; g0[c + 3] = ga.w;
    b0[c] = ba.x; b0[c + 1] = ba.y; b0[c + 2] = ba.z; b0[c + 3] = ba.w;
    g1[c] = gb.x; g1[c + 1] = gb.y; g1[c + 2] = gb.z; g1[c + 3] = gb.w;
    b1[c] = bb.x; b1[c + 1] = bb.y; b1[c + 2] = bb.z; b1[c + 3] = bb.w;
  }
}

template <int N, int NREAL, bool FINAL>
__device__ __forceinline__ void conv_epilogue(uint32_t tmem, const float* g0, const float* b0,
                                              const float* g1, const float* b1, const float* cb,
                                              uint8_t* act_hi, uint8_t* act_lo, float* red,
                                              __half* out_hi, __half* out_lo) {
  constexpr int NC = N / 2;
  const int w = warp_id(), q = w & 3, cg = w >> 2, lane = lane_id();
  const int c0 = cg * NC;
  const bool real = c0 < NREAL;            // conv3: the second column half is padding
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + c0;
  float x0[NC], x1[NC], y0[NC], y1[NC];
  if (NC == 32) {
    tmem_ld32(taddr, x0);
    tmem_ld32(taddr + N, y0);
    tmem_ld32(taddr + 128, x1);
    tmem_ld32(taddr + 128 + N, y1);
  } else {
    tmem_ldn<NC>(taddr, x0);
    tmem_ldn<NC>(taddr + N, y0);
    tmem_ldn<NC>(taddr + 128, x1);
    tmem_ldn<NC>(taddr + 128 + N, y1);
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {          // (hi*hi + lo*hi) + hi*lo
    x0[c] = __fadd_rn(x0[c], y0[c]);
    x1[c] = __fadd_rn(x1[c], y1[c]);
  }
  const int r0 = q * 32 + lane, r1 = 128 + r0;
  const int p0 = real ? interior_pixel(r0) : -1, p1 = real ? interior_pixel(r1) : -1;
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const float b = real ? cb[c0 + c] : 0.f;
    x0[c] = __fadd_rn(x0[c], b);
    x1[c] = __fadd_rn(x1[c], b);
    if (p0 >= 0) s += x0[c];
    if (p1 >= 0) s += x1[c];
  }
  constexpr float inv_n = 1.f / (float)(NREAL * kCnnHW);
  const float mean = cta_sum(s, red) * inv_n;
  float v = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const float d0 = x0[c] - mean, d1 = x1[c] - mean;
    if (p0 >= 0) v = fmaf(d0, d0, v);
    if (p1 >= 0) v = fmaf(d1, d1, v);
  }
  const float rstd = rsqrtf(cta_sum(v, red) * inv_n + 1e-5f);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int p = half ? p1 : p0;
    if (p < 0) continue;
    const float* x = half ? x1 : x0;
    const float* g = half ? g1 : g0;
    const float* bb = half ? b1 : b0;
    float y[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) y[c] = fmaxf(fmaf((x[c] - mean) * rstd, g[c], bb[c]), 0.f);
    if (!FINAL) {
      const int r = kActMargin + (half ? r1 : r0);
#pragma unroll
      for (int k = 0; k < NC / 8; ++k) {
        uint32_t hv[4], lv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float ya = y[8 * k + 2 * j], yb = y[8 * k + 2 * j + 1];
          const __half h0 = __float2half_rn(ya), h1 = __float2half_rn(yb);
          const __half l0 = __float2half_rn(__fsub_rn(ya, __half2float(h0)));
          const __half l1 = __float2half_rn(__fsub_rn(yb, __half2float(h1)));
          hv[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
          lv[j] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        const int c8 = c0 / 8 + k;
        const uint32_t off = r * 128 + ((c8 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(act_hi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4*>(act_lo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const __half h = __float2half_rn(y[c]);
        out_hi[(c0 + c) * kCnnHW + p] = h;
        out_lo[(c0 + c) * kCnnHW + p] = __float2half_rn(__fsub_rn(y[c], __half2float(h)));
      }
    }
  }
}

// One conv layer of the sample in the activation buffer: the MMAs (thread
// 0), the LN parameters fetched while they run, then the epilogue.
template <int C, int CIN, int TAPS, bool SPLIT, int NREAL, bool FINAL>
__device__ __forceinline__ bool conv_layer(uint32_t tmem, uint8_t* act_hi, uint8_t* act_lo,
                                           const uint8_t* w, uint64_t* dbar, uint32_t& phase,
                                           const float* __restrict__ lnf, int lg, int lb,
                                           const float* cb, float* red, __half* ohi,
                                           __half* olo) {
  constexpr int NC = C / 2;
  fence_proxy_async();
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    conv_mma<C, CIN, TAPS, SPLIT>(tmem, act_hi, act_lo, w);
    umma_commit(dbar);
  }
  float g0[NC], b0[NC], g1[NC], b1[NC];
  ln_params<C, NREAL>(lnf, lg, lb, g0, b0, g1, b1);
  const bool ok = __syncthreads_and(mbar_wait(dbar, phase & 1));
  ++phase;
  if (!ok) return false;
  asm volatile("tcgen05.fence::after_thread_sync;");
  conv_epilogue<C, NREAL, FINAL>(tmem, g0, b0, g1, b1, cb, act_hi, act_lo, red, ohi, olo);
  return true;
}

// The observation of one env (14 channels + 2 zero per interior pixel),
// one (pixel, 8-channel chunk) item per thread and pass: loaded into
// registers first, stored into the activation buffer's hi half later.
constexpr int kObsItems = 2 * kCnnHW;
__device__ __forceinline__ void obs_load(const __half* __restrict__ orow, uint32_t (*v)[4]) {
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = threadIdx.x + k * kTrunkWarps * 32;
    const int p = i >> 1, ch = i & 1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = ch * 8 + 2 * j;
      const bool in = i < kObsItems;
      const uint32_t a = in && c < 14 ? __half_as_ushort(orow[c * kCnnHW + p]) : 0u;
      const uint32_t b = in && c + 1 < 14 ? __half_as_ushort(orow[(c + 1) * kCnnHW + p]) : 0u;
      v[k][j] = a | (b << 16);
    }
  }
}

__device__ __forceinline__ void obs_store(const uint32_t (*v)[4], uint8_t* act_hi) {
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = threadIdx.x + k * kTrunkWarps * 32;
    if (i >= kObsItems) continue;
    const int p = i >> 1, ch = i & 1;
    const int r = kActMargin + (p / kCnnW + 1) * kCnnPW + (p % kCnnW + 1);
    *reinterpret_cast<uint4*>(act_hi + r * 128 + ((ch ^ (r & 7)) << 4)) =
        make_uint4(v[k][0], v[k][1], v[k][2], v[k][3]);
  }
}

__global__ void __launch_bounds__(kTrunkWarps * 32, 1)
k_cnn_trunk(const __half* __restrict__ obs, int obs_stride, int n, int n_seats,
            const uint8_t* __restrict__ pk, __half* __restrict__ out) {
  const CnnLayout L = cnn_layout(n_seats);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* act_hi = smem;
  uint8_t* act_lo = smem + kActBytes;
  uint8_t* wimg = smem + 2 * kActBytes;
  uint64_t* wbar = (uint64_t*)(wimg + ((L.wbytes + 15) & ~(size_t)15));
  uint64_t* dbar = wbar + 1;
  uint32_t* tmem_slot = (uint32_t*)(dbar + 1);
  float* red = (float*)(tmem_slot + 4);     // kTrunkWarps floats
  float* cb = red + kTrunkWarps;            // the 120 conv biases
  const float* lnf = (const float*)(pk + L.lnf);
  const int t = threadIdx.x;

  for (int i = t; i < 2 * kActBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  for (int i = t; i < LF_TOTAL - LF_CB0; i += blockDim.x) cb[i] = lnf[LF_CB0 + i];
  if (t == 0) {
    mbar_init(wbar, 1);
    mbar_init(dbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp_id() == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_proxy_async();
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  if (t == 0) {
    mbar_expect_tx(wbar, (uint32_t)L.wbytes);
    for (uint32_t o = 0; o < L.wbytes; o += 16384)
      bulk_load(wimg + o, pk + o, min((uint32_t)L.wbytes - o, 16384u), wbar);
  }
  bool ok = __syncthreads_and(mbar_wait(wbar, 0));
  uint32_t phase = 0;
  const int items = n * n_seats;
  static_assert(kObsItems <= 2 * kTrunkWarps * 32, "two observation items per thread");
  uint32_t ov[2][4];
  if ((int)blockIdx.x < items) {
    const int e = (int)blockIdx.x % n;
    obs_load(obs + (size_t)e * obs_stride, ov);
    obs_store(ov, act_hi);
  }
  for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
    const int seat = item / n, e = item - seat * n;
    const int next = item + (int)gridDim.x;
    __half* ohi = out + ((size_t)seat * 2 * n + e) * kCnnKP;
    __half* olo = out + ((size_t)seat * 2 * n + n + e) * kCnnKP;
    if (t < kCnnKP - kCnnKIn) {
      ohi[kCnnKIn + t] = __float2half_rn(0.f);
      olo[kCnnKIn + t] = __float2half_rn(0.f);
    }
    const uint8_t* w0 = wimg + L.c0 + (size_t)seat * kW0;
    ok = conv_layer<16, 16, 9, false, 16, false>(tmem, act_hi, act_lo, w0, dbar, phase, lnf,
                                                 LF_G0, LF_B0, cb, red, ohi, olo) &&
         conv_layer<32, 16, 9, true, 32, false>(tmem, act_hi, act_lo, wimg + L.c1, dbar, phase,
                                                lnf, LF_G1, LF_B1, cb + (LF_CB1 - LF_CB0), red,
                                                ohi, olo) &&
         conv_layer<64, 32, 9, true, 64, false>(tmem, act_hi, act_lo, wimg + L.c2, dbar, phase,
                                                lnf, LF_G2, LF_B2, cb + (LF_CB2 - LF_CB0), red,
                                                ohi, olo);
    if (!ok) break;
    // the next env's observation is fetched while the last layer runs and
    // stored once the layer's MMAs have read the activation buffer
    if (next < items) obs_load(obs + (size_t)(next % n) * obs_stride, ov);
    ok = conv_layer<16, 64, 1, true, 8, true>(tmem, act_hi, act_lo, wimg + L.c3, dbar, phase, lnf,
                                              LF_G3, LF_B3, cb + (LF_CB3 - LF_CB0), red, ohi,
                                              olo);
    if (ok && next < items) obs_store(ov, act_hi);
  }
  if (!ok && t == 0) {
    flag_error(QQT_DEV_TIMEOUT);
    // wait (bounded) for the weight copy and the MMAs of the last commit
    // before the shared memory and TMEM are given up
    mbar_wait(wbar, 0);
    if (phase > 0) mbar_wait(dbar, (phase - 1) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp_id() == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
  }
}

__host__ inline size_t cnn_trunk_smem(int n_seats) {
  const CnnLayout L = cnn_layout(n_seats);
  return 1024 + 2 * (size_t)kActBytes + ((L.wbytes + 15) & ~(size_t)15) + 128 +
         4 * (kTrunkWarps + (LF_TOTAL - LF_CB0));
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
  if (channels != 14 || hw != kCnnHW || n_seats < 1 || n_seats > 2) return 0;
  return cnn_layout(n_seats).total;
}

extern "C" int qqt_cnn_pack(const float* const* params_dev, int32_t n_players, int32_t channels,
                            int32_t hw, int32_t n_seats, const int32_t* pids, void* pack,
                            qqt_stream_t stream) {
  if (!params_dev || !pack || !pids || channels != 14 || hw != kCnnHW || n_seats < 1 ||
      n_seats > 2)
    return QQT_E_ARG;
  if (n_players != 2) return QQT_E_ARG;
  if ((uintptr_t)pack & 255) return QQT_E_ALIGN;
  for (int i = 0; i < 36; ++i)
    if (!params_dev[i]) return QQT_E_ARG;
  // stored channel k of seat s reads conv0 input column inv[k] (view permutation)
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
  const CnnLayout L = cnn_layout(n_seats);
  uint8_t* pk = (uint8_t*)pack;
  cudaStream_t st = (cudaStream_t)stream;
  CnnParams cp;
  for (int i = 0; i < 16; ++i) cp.p[i] = params_dev[i];
  // one thread per element of the largest item: the conv2 image (5 x 64 x 64)
  const int n_items = max(5 * 64 * 64, max(64 * kCnnHW, n_seats * 3 * 16 * 64));
  k_cnn_pack<<<(n_items + 255) / 256, 256, 0, st>>>(cp, n_seats, sc, pk);
  // Linear(1352 -> 128) + tail: an MLP pack with the identity column gather
  const MlpPack M = mlp_pack_layout(kCnnKIn, 1);
  SeatChannels id;
  memset(&id, 0, sizeof(id));
  for (int c = 0; c < 8; ++c) id.src[0][c] = c;
  uint8_t* mp = pk + L.mlp;
  const size_t total = (size_t)M.nt * M.kp;
  k_mlp_pack_w0<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      params_dev[16], kCnnKIn, M.kp, kCnnHW, 8, id, M.nt, (__half*)(mp + M.b_off));
  HeadParams hp;
  // q[] in the MLP parameter order: q[0] = shared.0.weight (index 16) ... q[19] = critic.2.bias
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
  k_mlp_pack_rest<<<(128 * 128 + 255) / 256, 256, 0, st>>>(hp, 1, (float*)(mp + M.f_off));
  k_mlp_pack_images<<<(192 * 128 + 255) / 256, 256, 0, st>>>(hp, mp + M.img_off);
  return launch_status();
}

// Flattened trunk outputs: [seat][hi, lo][N][1408] fp16.
extern "C" uint64_t qqt_cnn_work_bytes(int32_t n_envs, int32_t n_seats) {
  return (uint64_t)n_seats * 2 * (uint64_t)n_envs * kCnnKP * 2;
}


extern "C" int qqt_cnn_act(const void* pack, const void* obs, int32_t n_envs, int32_t obs_stride,
                           int32_t height, int32_t width, int32_t channels, int32_t n_seats,
                           const uint8_t* const* mm, int32_t mm_stride, const uint8_t* const* bm,
                           int32_t bm_stride, const float* u, int64_t* const* act,
                           int32_t act_stride, float* logp, float* value, float* logits,
                           void* work, qqt_stream_t stream) {
  if (!pack || !obs || !mm || !bm || !u || !act || !work || channels != 14) return QQT_E_ARG;
  if (n_envs <= 0 || n_seats < 1 || n_seats > 2 || height != kCnnH || width != kCnnW ||
      mm_stride < 5 || bm_stride < 2 || act_stride < 2)
    return QQT_E_ARG;
  if (obs_stride < channels * height * width) return QQT_E_ALIGN;
  if (((uintptr_t)pack & 255) || ((uintptr_t)work & 15)) return QQT_E_ALIGN;
  for (int s = 0; s < n_seats; ++s)
    if (!mm[s] || !bm[s] || !act[s]) return QQT_E_ARG;
  const CnnLayout L = cnn_layout(n_seats);
  const uint8_t* pk = (const uint8_t*)pack;
  cudaStream_t st = (cudaStream_t)stream;
  __half* out = (__half*)work;
  const size_t sm = cnn_trunk_smem(n_seats);
  cudaFuncSetAttribute(k_cnn_trunk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  const int items = n_envs * n_seats;
  k_cnn_trunk<<<min(items, sm_count()), kTrunkWarps * 32, sm, st>>>((const __half*)obs, obs_stride, n_envs,
                                                       n_seats, pk, out);
  const MlpPack M = mlp_pack_layout(kCnnKIn, 1);
  const uint8_t* mp = pk + L.mlp;
  CUtensorMap mb;
  if (!make_map(&mb, mp + M.b_off, (uint64_t)M.kp, (uint64_t)2 * M.nt, (uint64_t)M.kp * 2,
                (uint32_t)M.nt))
    return QQT_E_ARG;
  for (int s = 0; s < n_seats; ++s) {
    const __half* ahi = out + (size_t)s * 2 * n_envs * kCnnKP;
    const __half* alo = ahi + (size_t)n_envs * kCnnKP;
    CUtensorMap ma, malo;
    if (!make_map(&ma, ahi, kCnnKP, (uint64_t)n_envs, (uint64_t)kCnnKP * 2, kBM) ||
        !make_map(&malo, alo, kCnnKP, (uint64_t)n_envs, (uint64_t)kCnnKP * 2, kBM))
      return QQT_E_ARG;
    SeatOut io;
    io.mm[0] = mm[s];
    io.bm[0] = bm[s];
    io.act[0] = act[s];
    io.mm[1] = io.bm[1] = nullptr;
    io.act[1] = nullptr;
    const int rc = launch_mlp_fused<128, true>(ma, malo, mb, n_envs, M.kp / kBK,
                                               (const float*)(mp + M.f_off), mp + M.img_off, io,
                                               s, mm_stride, bm_stride, u, act_stride, logp,
                                               value, logits, st);
    if (rc != QQT_OK) return rc;
  }
  return launch_status();
}
