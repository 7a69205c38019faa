// MLP policy on the 5th-generation tensor cores, one fused kernel per 128
// env rows (train/model.py:121-153, 167-245).
//
// k_mlp_fused<NT>  (a cluster of ks CTAs per 128 envs, 576 threads each,
//                   NT = 128 x seats)
//   layer 1  split along K over the cluster: in CTA rank c, warp 0 lane 0
//            streams that rank's K tiles with TMA (no multicast): A = obs
//            tile [128 x 64] fp16, B = packed W0 (fp16 hi and lo halves of
//            the seat-permuted fp32 weights) [NT x 64]; warp 1 lane 0 issues
//            tcgen05.mma kind::f16 M=128 N=NT, two per K=16 step (A*Bhi +
//            A*Blo) into an fp32 TMEM accumulator; obs values are exact in
//            fp16 and the hi/lo split keeps W0's float32 precision.  Given
//            the rows' nonzero-tile flags, a K tile that is zero in all
//            128 rows is neither loaded nor multiplied (it adds exactly
//            zero).  Ranks
//            1..ks-1 copy their partial sums into their own shared memory
//            and arrive on an mbarrier of rank 0, whose epilogue adds them
//            in rank order (distributed shared memory reads).  The per-SM
//            TMA stream is what bounds layer 1, so the split divides it.
//   tail     (rank 0) the pipeline's shared memory is reused: one bulk copy
//            brings the pre-swizzled fp16 hi/lo images of shared.3
//            (128x128) and the three head hidden layers (192x128).  16
//            epilogue warps give each row four threads (TMEM lane quadrant
//            x column quarter): tcgen05.ld the quarter, +bias, LayerNorm
//            (the row sums cross the four threads through scratch columns
//            of the row's own TMEM lane), ReLU, split into fp16 hi/lo and
//            store it as the next MMA's A operand (128-byte swizzled
//            K-major).  Each of the two remaining layers is 8 K steps x 3
//            MMAs (Ahi*Whi + Ahi*Wlo + Alo*Whi), which keeps the products at
//            float32 accuracy.  Each thread takes a share of the 192 head
//            units (the four shares hold about equal numbers of output
//            multiply-adds) and forms partial output logits (5 move, 2
//            bomb, 1 value); the
//            first quarter's thread sums the four, masks with float32's
//            lowest value, samples by inverse CDF and writes the
//            log-probability and value.
// The CNN policy (policy_cnn.cu) reuses this kernel with SPLIT_A for its
// Linear(1352 -> 128) and the same tail.
//
// Every mbarrier wait is bounded; on expiry the CTA raises QQT_DEV_TIMEOUT,
// waits (bounded) for the copies and MMAs it issued, frees its TMEM and
// returns.  Branch decisions after a wait are made uniform over the epilogue
// warps (barrier with an AND reduction), and every thread reaches the
// closing cluster barrier, so no CTA leaves while another reads its shared
// memory.

#include <cuda.h>

#include <atomic>

#include "qqt_common.cuh"

namespace qqt {

constexpr int kBM = 128;          // env rows per CTA
constexpr int kBK = 64;           // K elements per stage (128 bytes of fp16)
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false (and the timeout flag) when the limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t limit = kWaitLimit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  flag_error(QQT_DEV_TIMEOUT);
  return false;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Four rows (y0..y3) of columns x..x+63 of a tensor map whose box is one
// row high, landing as a four-row box at dst (TMA tile::gather4).
__device__ __forceinline__ void tma_gather4(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y0, int y1, int y2, int y3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Generic-proxy shared-memory writes -> visible to the tensor cores.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte offset of element (n, k) in a K-major operand image of `nrows` rows
// and K = 128 stored as two 64-wide K blocks with the 128-byte swizzle
// (row n at n*128 bytes, 16-byte chunk c at chunk c ^ (n % 8)).
__host__ __device__ __forceinline__ uint32_t sw128_off(int n, int k, int nrows) {
  return (uint32_t)((k >> 6) * nrows * 128 + n * 128 + ((((k & 63) >> 3) ^ (n & 7)) << 4) +
                    (k & 7) * 2);
}

// K-major operand tile with 128-byte swizzle: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address
  d |= (uint64_t)1 << 16;                // leading byte offset (16 B, unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;      // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: fp16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Two 32-column loads (columns a .. a+31 and b .. b+31 of the warp's lanes)
// with one wait, so the second load's latency overlaps the first's.
__device__ __forceinline__ void tmem_ld32x2(uint32_t a, uint32_t b, float* x, float* y) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(a), "r"(b)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    x[i] = __uint_as_float(r[i]);
    y[i] = __uint_as_float(r[32 + i]);
  }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------ pack layout

// Pack (bytes): [B fp16: 2 x NT x KP] [f32 params] [tail operand images]
// [the same images as two row halves, for the SM-pair kernel]
struct MlpPack {
  int kp, nt, n_seats;
  size_t b_off, f_off, img_off, pair_off, total;
};

// Tail operand images (bytes from img_off), each 128-byte swizzled K-major,
// K = 128, fp16 hi then lo: shared.3 [128 out x 128 in], then the three head
// hidden layers stacked [192 x 128] (move 0-63, bomb 64-127, critic 128-191).
constexpr uint32_t kImgW1 = 0, kImgW1Bytes = 128 * 128 * 2;          // per hi / lo
constexpr uint32_t kImgH0 = 2 * kImgW1Bytes, kImgH0Bytes = 192 * 128 * 2;
constexpr uint32_t kImgBytes = kImgH0 + 2 * kImgH0Bytes;             // 160 KB

// f32 parameter block offsets (floats)
enum {
  F_B0 = 0,                       // [NT] first-layer bias per seat column
  F_LN1G = F_B0 + 256, F_LN1B = F_LN1G + 128,
  F_W1 = F_LN1B + 128,            // [128 in][128 out] (transposed)
  F_B1 = F_W1 + 128 * 128,
  F_LN2G = F_B1 + 128, F_LN2B = F_LN2G + 128,
  F_HW0 = F_LN2B + 128,           // [128 in][192 hidden] (transposed; move, bomb, critic)
  F_HB0 = F_HW0 + 3 * 64 * 128,   // [192]
  F_HW2 = F_HB0 + 3 * 64,         // [8][64] rows: 5 move, 2 bomb, 1 value
  F_HB2 = F_HW2 + 8 * 64,         // [8]
  F_TOTAL = F_HB2 + 8
};

__host__ __device__ inline MlpPack mlp_pack_layout(int k_in, int n_seats) {
  MlpPack p;
  p.kp = (k_in + kBK - 1) / kBK * kBK;
  p.nt = 128 * n_seats;
  p.n_seats = n_seats;
  p.b_off = 0;
  p.f_off = ((size_t)2 * p.nt * p.kp * 2 + 255) / 256 * 256;
  p.img_off = (p.f_off + (size_t)F_TOTAL * 4 + 1023) / 1024 * 1024;
  p.pair_off = p.img_off + kImgBytes;
  p.total = p.pair_off + kImgBytes;
  return p;
}

// One thread per packed weight element: column gather by the seat's view
// permutation, then the fp16 hi / lo split.
struct SeatChannels {
  int32_t src[2][64];   // W0 column block used by stored channel c of seat s
};

__global__ void k_mlp_pack_w0(const float* __restrict__ w0, int k_in, int kp, int hw, int channels,
                              SeatChannels sc, int nt, __half* __restrict__ b) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)nt * kp;
  if (i >= total) return;
  const int row = (int)(i / kp), k = (int)(i % kp);
  float wv = 0.f;
  if (k < k_in) {
    const int seat = row / 128, r = row % 128;
    const int ch = k / hw, cell = k - ch * hw;
    const int src = sc.src[seat][ch] * hw + cell;
    wv = w0[(size_t)r * k_in + src];
  }
  const __half hi = __float2half_rn(wv);
  const __half lo = __float2half_rn(__fsub_rn(wv, __half2float(hi)));
  b[(size_t)row * kp + k] = hi;
  b[(size_t)nt * kp + (size_t)row * kp + k] = lo;
}

struct HeadParams {
  const float *b0, *ln1g, *ln1b, *w1, *b1, *ln2g, *ln2b;
  const float *mw0, *mb0, *mw2, *mb2, *bw0, *bb0, *bw2, *bb2, *cw0, *cb0, *cw2, *cb2;
};

__global__ void k_mlp_pack_rest(HeadParams hp, int n_seats, float* __restrict__ f) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 128 * n_seats) f[F_B0 + i] = hp.b0[i % 128];
  if (i < 128) {
    f[F_LN1G + i] = hp.ln1g[i];
    f[F_LN1B + i] = hp.ln1b[i];
    f[F_B1 + i] = hp.b1[i];
    f[F_LN2G + i] = hp.ln2g[i];
    f[F_LN2B + i] = hp.ln2b[i];
  }
  if (i < 128 * 128) {
    const int o = i / 128, k = i % 128;                 // w1 is [out][in]
    f[F_W1 + k * 128 + o] = hp.w1[i];
  }
  if (i < 64 * 128) {
    const int o = i / 128, k = i % 128;                 // head weights [64][128]
    f[F_HW0 + k * 192 + o] = hp.mw0[i];
    f[F_HW0 + k * 192 + 64 + o] = hp.bw0[i];
    f[F_HW0 + k * 192 + 128 + o] = hp.cw0[i];
  }
  if (i < 64) {
    f[F_HB0 + i] = hp.mb0[i];
    f[F_HB0 + 64 + i] = hp.bb0[i];
    f[F_HB0 + 128 + i] = hp.cb0[i];
  }
  if (i < 8 * 64) {
    const int r = i / 64, c = i % 64;
    float v;
    if (r < 5) v = hp.mw2[r * 64 + c];
    else if (r < 7) v = hp.bw2[(r - 5) * 64 + c];
    else v = hp.cw2[c];
    f[F_HW2 + i] = v;
  }
  if (i < 8) f[F_HB2 + i] = i < 5 ? hp.mb2[i] : (i < 7 ? hp.bb2[i - 5] : hp.cb2[0]);
}

// fp16 hi / lo split of shared.3 and the head hidden layers into the
// swizzled operand images, one thread per (row, k).
__global__ void k_mlp_pack_images(HeadParams hp, uint8_t* __restrict__ img) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 192 * 128) return;
  const int n = i >> 7, k = i & 127;
  if (n < 128) {
    const float v = hp.w1[n * 128 + k];                  // [out][in]: K-major already
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    *reinterpret_cast<__half*>(img + kImgW1 + sw128_off(n, k, 128)) = hi;
    *reinterpret_cast<__half*>(img + kImgW1 + kImgW1Bytes + sw128_off(n, k, 128)) = lo;
  }
  const float v = n < 64 ? hp.mw0[n * 128 + k]
                         : (n < 128 ? hp.bw0[(n - 64) * 128 + k] : hp.cw0[(n - 128) * 128 + k]);
  const __half hi = __float2half_rn(v);
  const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
  *reinterpret_cast<__half*>(img + kImgH0 + sw128_off(n, k, 192)) = hi;
  *reinterpret_cast<__half*>(img + kImgH0 + kImgH0Bytes + sw128_off(n, k, 192)) = lo;
}

// ---------------------------------------------------------------- heads

// The sampling inputs of one row: legal-move bits (bit k: move k, bits 5
// and 6: bomb 0 and 1) and the two uniforms.  The epilogue loads them before
// layer 1 completes, so their latency stays off the tail's critical path.
struct SampleIn {
  uint32_t legal;
  float um, ub;
};

__device__ __forceinline__ SampleIn sample_load(int row, int seat, int n_rows,
                                                const uint8_t* __restrict__ mm, int mm_stride,
                                                const uint8_t* __restrict__ bm, int bm_stride,
                                                const float* __restrict__ u) {
  const uint8_t* mrow = mm + (size_t)row * mm_stride;
  const uint8_t* brow = bm + (size_t)row * bm_stride;
  SampleIn in;
  uint32_t b = 0;
#pragma unroll
  for (int k = 0; k < 5; ++k) b |= (mrow[k] ? 1u : 0u) << k;
  b |= (brow[0] ? 1u : 0u) << 5;
  b |= (brow[1] ? 1u : 0u) << 6;
  in.legal = b;
  in.um = u[((size_t)seat * n_rows + row) * 2];
  in.ub = u[((size_t)seat * n_rows + row) * 2 + 1];
  return in;
}

// Logits z (5 move, 2 bomb, value) of one row -> masked categorical samples
// (inverse CDF: a = #{k : u * S > cs_k} over exp(z - max z)), joint
// log-prob, value; masked logits take float32's lowest value
// (train/model.py:204-245).
__device__ __forceinline__ void sample_write(const float* z, int row, int seat, int n_rows,
                                             const SampleIn& in, int64_t* __restrict__ act,
                                             int act_stride, float* __restrict__ logp_out,
                                             float* __restrict__ value_out,
                                             float* __restrict__ logits_out) {
  if (logits_out) {
    float* lo = logits_out + ((size_t)seat * n_rows + row) * 8;
#pragma unroll
    for (int o = 0; o < 8; ++o) lo[o] = z[o];
  }
  const float lowest = -3.402823466e38f;
  float zm[5], cs[5];
  float mx = lowest;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    zm[k] = (in.legal >> k) & 1u ? z[k] : lowest;
    mx = fmaxf(mx, zm[k]);
  }
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    tot += expf(zm[k] - mx);
    cs[k] = tot;
  }
  const float um = in.um * tot;
  int am = 0;
#pragma unroll
  for (int k = 0; k < 5; ++k) am += um > cs[k];
  am = min(am, 4);
  float zam = zm[0];
#pragma unroll
  for (int k = 1; k < 5; ++k) zam = am == k ? zm[k] : zam;
  const float lpm = zam - mx - logf(tot);
  const float zb0 = (in.legal >> 5) & 1u ? z[5] : lowest;
  const float zb1 = (in.legal >> 6) & 1u ? z[6] : lowest;
  const float mb = fmaxf(zb0, zb1);
  const float e0 = expf(zb0 - mb), s2 = e0 + expf(zb1 - mb);
  const float ub = in.ub * s2;
  const int ab = ub > e0 ? 1 : 0;
  const float lpb = (ab ? zb1 : zb0) - mb - logf(s2);
  act[(size_t)row * act_stride] = am;
  act[(size_t)row * act_stride + 1] = ab;
  if (logp_out) logp_out[(size_t)seat * n_rows + row] = lpm + lpb;
  if (value_out) value_out[(size_t)seat * n_rows + row] = z[7];
}

// Logits z of one row scored against the row's recorded actions (the
// reference's evaluate, train/model.py:247-256): each head's masked logits
// (illegal entries at float32's lowest value) minus their logsumexp
// (max + log of the shifted sum), logp = lz_move[a_move] + lz_bomb[a_bomb],
// entropy = -sum(max(lz, lowest) * exp(lz)) over both heads, value.
__device__ __forceinline__ void score_write(const float* z, int row,
                                            const uint8_t* __restrict__ mm, int mm_stride,
                                            const uint8_t* __restrict__ bm, int bm_stride,
                                            const int64_t* __restrict__ act, int act_stride,
                                            float* __restrict__ logp_out,
                                            float* __restrict__ ent_out,
                                            float* __restrict__ value_out) {
  const float lowest = -3.402823466e38f;
  const uint8_t* mrow = mm + (size_t)row * mm_stride;
  const uint8_t* brow = bm + (size_t)row * bm_stride;
  float zm[5], mx = lowest;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    zm[k] = mrow[k] ? z[k] : lowest;
    mx = fmaxf(mx, zm[k]);
  }
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 5; ++k) tot += expf(zm[k] - mx);
  const float lse_m = logf(tot) + mx;
  const float zb[2] = {brow[0] ? z[5] : lowest, brow[1] ? z[6] : lowest};
  const float mb = fmaxf(zb[0], zb[1]);
  const float lse_b = logf(expf(zb[0] - mb) + expf(zb[1] - mb)) + mb;
  long long am = act[(size_t)row * act_stride], ab = act[(size_t)row * act_stride + 1];
  if (am < 0 || am > 4 || ab < 0 || ab > 1) {
    flag_error(QQT_DEV_BAD_ACTION);
    am = 0;
    ab = 0;
  }
  float lpm = 0.f, ent = 0.f;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const float lz = zm[k] - lse_m;
    lpm = am == k ? lz : lpm;
    ent += fmaxf(lz, lowest) * expf(lz);
  }
  float lpb = 0.f, entb = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float lz = zb[k] - lse_b;
    lpb = ab == k ? lz : lpb;
    entb += fmaxf(lz, lowest) * expf(lz);
  }
  logp_out[row] = lpm + lpb;
  ent_out[row] = -ent - entb;
  value_out[row] = z[7];
}

// Training forward outputs (k_mlp_fused<128, false, true>): the pre-LN
// activations of both trunk layers [n_rows][128] and the entropy per row.
struct TrainOut {
  float* h1;
  float* h2;
  float* ent;
  const int64_t* idx;    // optional: row r of the minibatch is row idx[r] of the A map
  int n_src;             // rows of the A map (idx bounds)
};

// ------------------------------------------------------------ fused MLP

struct SeatOut {
  const uint8_t* mm[2];
  const uint8_t* bm[2];
  int64_t* act[2];
};

// SPLIT_A: the A operand is an fp32 activation given as fp16 hi and lo
// halves (two tensor maps); each K step then issues the third product
// A_lo * W_hi.  Without it A is the exact fp16 observation.
template <int NT, bool SPLIT_A = false>
struct FusedCfg {
  static constexpr int kStages = (NT == 128 && !SPLIT_A) ? 4 : (NT == 128 ? 3 : 2);
  static constexpr int kABytes = kBM * kBK * 2;         // one of hi / lo
  static constexpr int kAAll = kABytes * (SPLIT_A ? 2 : 1);
  static constexpr int kBBytes = NT * kBK * 2;          // one of hi / lo
  static constexpr int kStageBytes = kAAll + 2 * kBBytes;
  static constexpr int kPipeBytes = kStages * kStageBytes;
  // tail layout inside the (reused) pipeline region
  static constexpr int kW1 = 0;                         // shared.3 hi, lo
  static constexpr int kH0 = (int)kImgH0;               // head hidden hi, lo
  static constexpr int kAct = (int)kImgBytes;           // activation operand hi, lo
  static constexpr int kActBytes = kBM * 128 * 2;       // one of hi / lo
  static constexpr int kTailBytes = kAct + 2 * kActBytes;
  static constexpr int kRegion = kPipeBytes > kTailBytes ? kPipeBytes : kTailBytes;
  static constexpr int kSmem = kRegion + 1024 /*align*/ + 256 /*barriers*/ + 512 /*row ids*/;
  // split-K partial sums of a non-leader CTA: [seat][128 rows][128] fp32 at
  // the start of its (drained) pipeline region
  static constexpr int kPartBytes = (NT / 128) * kBM * 128 * 4;
  static constexpr uint32_t kTmemCols = 512;            // leader
  // layer 1: one seat accumulates A W_hi and A W_lo in columns [0, 128) and
  // [128, 256) (one N = 256 MMA over the stacked hi / lo weight rows, so
  // the A tile is read once per K step); two seats accumulate both
  // products into the seat's 128 columns
  static constexpr uint32_t kL1Cols = NT == 128 ? 256 : NT;
  static constexpr uint32_t kColH = NT;                 // head hidden accumulator (192 cols)
  static constexpr uint32_t kColScr = NT + 192;         // row-exchange scratch (48 cols)
};
static_assert(FusedCfg<128>::kSmem <= 232448 && FusedCfg<256>::kSmem <= 232448 &&
                  FusedCfg<128, true>::kSmem <= 232448,
              "fused MLP shared memory over the per-CTA limit");
// barriers (full, empty: kStages each; accb, wbar, abar, dbar, pready), TMEM
// slot and abort flag below byte 192 of the barrier block, the K-tile flags
// in [192, 256), the gathered row ids after it
static_assert((2 * FusedCfg<128>::kStages + 5) * 8 + 8 <= 192 &&
                  (2 * FusedCfg<256>::kStages + 5) * 8 + 8 <= 192 &&
                  (2 * FusedCfg<128, true>::kStages + 5) * 8 + 8 <= 192,
              "fused barrier block");
static_assert(FusedCfg<256>::kColScr + 48 <= FusedCfg<256>::kTmemCols &&
                  FusedCfg<128>::kColScr + 48 <= FusedCfg<128>::kTmemCols,
              "TMEM columns");
static_assert(FusedCfg<128>::kPartBytes <= FusedCfg<128>::kPipeBytes &&
                  FusedCfg<256>::kPartBytes <= FusedCfg<256>::kPipeBytes &&
                  FusedCfg<128, true>::kPartBytes <= FusedCfg<128, true>::kPipeBytes,
              "split-K partials fit the pipeline region");

// Block: warp 0 TMA producer, warp 1 MMA issuer, 16 epilogue warps.  Epilogue
// warp e = warp - 2 owns TMEM lane quadrant warp % 4 (32 rows) and column
// quarter e / 4 (32 of a layer's 128 columns): four threads per row.
constexpr int kEpiWarps = 16;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kMlpThreads = 64 + kEpiThreads;
constexpr int kMaxSplitK = 8;

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr),
               "r"(__float_as_uint(v))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                   taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Barrier of the 16 epilogue warps (named barrier 1).
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

// Barrier of the 16 epilogue warps that also ANDs a flag over them, so that
// every epilogue warp takes the same branch after a bounded wait.
__device__ __forceinline__ bool epi_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

// The four values of a row (one per column quarter, four warps) through the
// row's TMEM lane: each thread writes its value into column scr + quarter,
// then, after the epilogue barrier, reads all four.
__device__ __forceinline__ void row_exchange4(uint32_t scr, int quarter, float v, float* p) {
  tmem_st1(scr + quarter, v);
  asm volatile("tcgen05.fence::before_thread_sync;");
  epi_sync();
  asm volatile("tcgen05.fence::after_thread_sync;");
  tmem_ld4(scr, p);
}

// Barrier of the four epilogue warps of k_mlp_fused / k_mlp_pair that share
// TMEM lane quadrant warp % 4 (one warp per column quarter, so the four
// threads of each of those 32 rows): named barriers 2..5.
__device__ __forceinline__ void quad_sync() {
  switch (warp_id() & 3) {   // constant barrier ids
    case 0: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
    default: asm volatile("bar.sync 5, 128;" ::: "memory"); break;
  }
}

// row_exchange4 among the four threads of a row only (quad_sync).
__device__ __forceinline__ void row_exchange4_quad(uint32_t scr, int quarter, float v, float* p) {
  tmem_st1(scr + quarter, v);
  asm volatile("tcgen05.fence::before_thread_sync;");
  quad_sync();
  asm volatile("tcgen05.fence::after_thread_sync;");
  tmem_ld4(scr, p);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}
// Bounded wait with cluster-scope acquire (arrivals from other CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  flag_error(QQT_DEV_TIMEOUT);
  return false;
}

// Head output layers over head hidden units U0 .. U0+NU-1 (inside one head;
// TMEM columns hcol + U0 ..): +bias, ReLU, then the head's output rows
// (train/model.py:167-245: move_head.2 / bomb_head.2 / critic.2) into this
// thread's partial logits z (5 move, 2 bomb, 1 value).
template <int U0, int NU>
__device__ __forceinline__ void head_out_chunk(uint32_t hcol, const float* __restrict__ f,
                                               float* z) {
  static_assert(NU == 8 || NU == 16 || NU == 32, "chunk width");
  static_assert((U0 >> 6) == ((U0 + NU - 1) >> 6), "a chunk lies inside one head");
  float h[NU];
  if constexpr (NU == 8) tmem_ld8(hcol + U0, h);
  else if constexpr (NU == 16) tmem_ld16(hcol + U0, h);
  else tmem_ld32(hcol + U0, h);
  constexpr int head = U0 >> 6, uu = U0 & 63;
  constexpr int o_lo = head == 0 ? 0 : (head == 1 ? 5 : 7);
  constexpr int o_hi = head == 0 ? 5 : (head == 1 ? 7 : 8);
#pragma unroll
  for (int i = 0; i < NU; i += 4) {
    const float4 hb = __ldg(reinterpret_cast<const float4*>(f + F_HB0 + U0 + i));
    h[i] = fmaxf(__fadd_rn(h[i], hb.x), 0.f);
    h[i + 1] = fmaxf(__fadd_rn(h[i + 1], hb.y), 0.f);
    h[i + 2] = fmaxf(__fadd_rn(h[i + 2], hb.z), 0.f);
    h[i + 3] = fmaxf(__fadd_rn(h[i + 3], hb.w), 0.f);
  }
#pragma unroll
  for (int o = o_lo; o < o_hi; ++o)
#pragma unroll
    for (int i = 0; i < NU; i += 4) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(f + F_HW2 + o * 64 + uu + i));
      z[o] = fmaf(wv.x, h[i], z[o]);
      z[o] = fmaf(wv.y, h[i + 1], z[o]);
      z[o] = fmaf(wv.z, h[i + 2], z[o]);
      z[o] = fmaf(wv.w, h[i + 3], z[o]);
    }
}

// The four threads of a row split the 512 output multiply-adds (64 move
// units x 5 + 64 bomb units x 2 + 64 value units x 1) about evenly: units
// 0-23 (120), 24-47 (120), 48-87 (128), 88-191 (144).  `quarter` is
// warp-uniform, so every TMEM load stays warp-collective.
__device__ __forceinline__ void head_out_quarter(uint32_t hcol, int quarter,
                                                 const float* __restrict__ f, float* z) {
  switch (quarter) {
    case 0:
      head_out_chunk<0, 16>(hcol, f, z);
      head_out_chunk<16, 8>(hcol, f, z);
      break;
    case 1:
      head_out_chunk<24, 8>(hcol, f, z);
      head_out_chunk<32, 16>(hcol, f, z);
      break;
    case 2:
      head_out_chunk<48, 16>(hcol, f, z);
      head_out_chunk<64, 16>(hcol, f, z);
      head_out_chunk<80, 8>(hcol, f, z);
      break;
    default:
      head_out_chunk<88, 8>(hcol, f, z);
      head_out_chunk<96, 32>(hcol, f, z);
      head_out_chunk<128, 32>(hcol, f, z);
      head_out_chunk<160, 32>(hcol, f, z);
      break;
  }
}

// Byte offset of float4 chunk c (of 32) of row r in a [128][128] fp32
// partial-sum block; the chunk index is XOR-swizzled by the row so that a
// warp's 32 rows hit distinct bank groups.
__device__ __forceinline__ uint32_t part_off(int r, int c) {
  return (uint32_t)(r * 512 + ((c ^ (r & 31)) << 4));
}

// x[32] (+bias) -> LayerNorm over the row's 128 columns (this thread holds
// columns 32q..32q+31; the sums go through the TMEM row exchange) -> affine
// -> ReLU (train/model.py:121-153).
// pre (optional): the thread's 32 pre-LayerNorm values (bias included) are
// also written there (the training forward keeps them for the backward).
__device__ __forceinline__ void bias_ln_relu_quarter(float* x, int q, uint32_t scr,
                                                     const float* __restrict__ bias,
                                                     const float* __restrict__ g,
                                                     const float* __restrict__ b,
                                                     float* __restrict__ pre = nullptr) {
  const int c0 = 32 * q;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + c0 + i));
    x[i] = __fadd_rn(x[i], bb.x);
    x[i + 1] = __fadd_rn(x[i + 1], bb.y);
    x[i + 2] = __fadd_rn(x[i + 2], bb.z);
    x[i + 3] = __fadd_rn(x[i + 3], bb.w);
    if (pre) *reinterpret_cast<float4*>(pre + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) s4[j] += x[i + j];
  }
  float p[4];
  row_exchange4_quad(scr, q, (s4[0] + s4[1]) + (s4[2] + s4[3]), p);
  const float mean = ((p[0] + p[1]) + (p[2] + p[3])) * (1.f / 128.f);
  float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; i += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = x[i + j] - mean;
      v4[j] = fmaf(d, d, v4[j]);
    }
  row_exchange4_quad(scr + 4, q, (v4[0] + v4[1]) + (v4[2] + v4[3]), p);
  const float rstd = rsqrtf(((p[0] + p[1]) + (p[2] + p[3])) * (1.f / 128.f) + 1e-5f);
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 gg = __ldg(reinterpret_cast<const float4*>(g + c0 + i));
    const float4 be = __ldg(reinterpret_cast<const float4*>(b + c0 + i));
    x[i] = fmaxf(fmaf((x[i] - mean) * rstd, gg.x, be.x), 0.f);
    x[i + 1] = fmaxf(fmaf((x[i + 1] - mean) * rstd, gg.y, be.y), 0.f);
    x[i + 2] = fmaxf(fmaf((x[i + 2] - mean) * rstd, gg.z, be.z), 0.f);
    x[i + 3] = fmaxf(fmaf((x[i + 3] - mean) * rstd, gg.w, be.w), 0.f);
  }
}

// Columns 32q..32q+31 of row r of the activation operand: fp16 hi and lo
// images, 16-byte stores.
__device__ __forceinline__ void store_split_quarter(const float* x, uint8_t* a_hi, uint8_t* a_lo,
                                                    int r, int q) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // packed conversions: element 2j in the low half, 2j+1 in the high
      const float v0 = x[8 * c + 2 * j], v1 = x[8 * c + 2 * j + 1];
      const __half2 h = __floats2half2_rn(v0, v1);
      const float2 hf = __half22float2(h);
      const __half2 l = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
      hv[j] = *reinterpret_cast<const uint32_t*>(&h);
      lv[j] = *reinterpret_cast<const uint32_t*>(&l);
    }
    const uint32_t off = sw128_off(r, 32 * q + 8 * c, kBM);
    *reinterpret_cast<uint4*>(a_hi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(a_lo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

// D[tmem] (+)= A * W over K = 128 with the three-term fp16 split.
__device__ __forceinline__ void umma_split_k128(uint32_t d_tmem, const uint8_t* a_hi,
                                                const uint8_t* a_lo, const uint8_t* w_hi,
                                                const uint8_t* w_lo, int w_rows, uint32_t idesc) {
  const uint64_t ah = sw128_desc(a_hi), al = sw128_desc(a_lo);
  const uint64_t wh = sw128_desc(w_hi), wl = sw128_desc(w_lo);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t oa = (uint64_t)(((kk >> 2) * kBM * 128 + (kk & 3) * 32) >> 4);
    const uint64_t ow = (uint64_t)(((kk >> 2) * w_rows * 128 + (kk & 3) * 32) >> 4);
    umma_f16(d_tmem, ah + oa, wh + ow, idesc, kk > 0 ? 1u : 0u);
    umma_f16(d_tmem, ah + oa, wl + ow, idesc, 1u);
    umma_f16(d_tmem, al + oa, wh + ow, idesc, 1u);
  }
}

// ---- layer-1 K tiles that hold a nonzero observation entry
//
// The caller may pass, per observation row, four 32-bit words that flag the
// row's K tiles (64 fp16 entries each) holding a nonzero: tile t is flagged
// by bit min(t >> 2, 31) of word t & 3 (bit 31 also stands for every tile
// past 127).  A tile that is zero in every row of a CTA's row tile adds
// exactly zero to each layer-1 accumulator, so the CTA neither loads it nor
// issues its MMAs; the tiles that do run keep their order, so the sums are
// the ones the full pass produces.  The flags may over-report (a flagged
// zero tile costs time only); they must never miss a nonzero.  Without
// flags every tile runs.
// Bring a TMA descriptor (a __grid_constant__ kernel parameter) into the
// descriptor cache ahead of the first copy that uses it.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ bool ktile_on(const uint4& m, int t) {
  const int q = t & 3;
  const uint32_t w = q == 0 ? m.x : (q == 1 ? m.y : (q == 2 ? m.z : m.w));
  return (w >> min(t >> 2, 31)) & 1u;
}

// Warps 2..5: warp 2 + q ORs the flags of rows r0 + q*32 + lane (+128, ...)
// below min(r1, n_rows) into part[q]; no flags: every bit set.
__device__ __forceinline__ void ktile_flags_part(const uint4* __restrict__ tiles, int r0, int r1,
                                                 int n_rows, uint4* part) {
  const int q = warp_id() - 2;
  uint4 m = make_uint4(~0u, ~0u, ~0u, ~0u);
  if (tiles) {
    m = make_uint4(0, 0, 0, 0);
    const int lim = min(r1, n_rows);
    for (int r = r0 + q * 32 + lane_id(); r < lim; r += 128) {
      const uint4 v = tiles[r];
      m.x |= v.x;
      m.y |= v.y;
      m.z |= v.z;
      m.w |= v.w;
    }
    m.x = __reduce_or_sync(QQT_FULL, m.x);
    m.y = __reduce_or_sync(QQT_FULL, m.y);
    m.z = __reduce_or_sync(QQT_FULL, m.z);
    m.w = __reduce_or_sync(QQT_FULL, m.w);
  }
  if (lane_id() == 0) part[q] = m;
}

__device__ __forceinline__ uint4 ktile_flags(const uint4* part) {
  uint4 m = part[0];
#pragma unroll
  for (int q = 1; q < 4; ++q) {
    m.x |= part[q].x;
    m.y |= part[q].y;
    m.z |= part[q].z;
    m.w |= part[q].w;
  }
  return m;
}

// The flags as a 64-bit mask over the first 64 K tiles, for every lane of
// the calling warp (two ballots); rows of more than 64 tiles run them all.
__device__ __forceinline__ uint64_t ktile_mask(const uint4* part, int k_tiles) {
  const uint4 m = ktile_flags(part);
  const int l = lane_id();
  const uint32_t lo = __ballot_sync(QQT_FULL, l < k_tiles && ktile_on(m, l));
  const uint32_t hi = __ballot_sync(QQT_FULL, l + 32 < k_tiles && ktile_on(m, l + 32));
  return k_tiles > 64 ? ~0ull : (((uint64_t)hi << 32) | lo);
}

__device__ __forceinline__ bool ktile_in(uint64_t mask, int t) {
  return t >= 64 || ((mask >> t) & 1ull);
}

// Tiles a CTA runs out of [kt0, kt1), visited from tile `first`: that one
// always (so the accumulators are written even if every flag is clear),
// then the flagged ones.
__device__ __forceinline__ int ktile_count(uint64_t mask, int kt0, int kt1, int first) {
  if (kt1 > 64 || mask == ~0ull) return kt1 - kt0;
  const int n = kt1 - kt0;
  const uint64_t range = (n >= 64 ? ~0ull : ((1ull << n) - 1)) << kt0;
  return __popcll(mask & range) + (ktile_in(mask, first) ? 0 : 1);
}

// One cluster of ks CTAs (launched with cluster dimension ks, 1 <= ks <= 8)
// serves 128 env rows.  Layer 1 is split along K: CTA rank c accumulates K
// tiles [c*kt/ks, (c+1)*kt/ks) into its own TMEM; the other ranks copy their
// partial sums into their own shared memory and signal the rank-0 CTA, whose
// epilogue adds them (rank order) to its own while applying LN1, then runs
// the rest of the network alone.  ks = 1 is a plain one-CTA launch.
template <int NT, bool SPLIT_A, bool TRAIN>
__global__ void __launch_bounds__(kMlpThreads, 1)
k_mlp_fused(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_alo,
            const __grid_constant__ CUtensorMap tm_b, int n_rows, int k_tiles,
            const float* __restrict__ f, const uint8_t* __restrict__ img, SeatOut io, int seat0,
            int mm_stride, int bm_stride, const float* __restrict__ u, int act_stride,
            float* __restrict__ logp_out, float* __restrict__ value_out,
            float* __restrict__ logits_out, TrainOut tr, uint32_t test_wait,
            const uint4* __restrict__ tiles) {
  static_assert(!TRAIN || (NT == 128 && !SPLIT_A), "training forward: one seat, fp16 rows");
  using G = FusedCfg<NT, SPLIT_A>;
  constexpr int S = NT / 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + G::kRegion);
  uint64_t* empty = full + G::kStages;
  uint64_t* accb = empty + G::kStages;    // layer-1 accumulator complete
  uint64_t* wbar = accb + 1;              // tail weight images landed
  uint64_t* abar = wbar + 1;              // activation operand written (512 arrivals)
  uint64_t* dbar = abar + 1;              // tail MMA group complete
  uint64_t* pready = dbar + 1;            // split-K partials of the other ranks written
  uint32_t* tmem_slot = (uint32_t*)(pready + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  uint4* kpart = (uint4*)(smem + G::kRegion + 192);   // K-tile flags, one word set per warp
  const int warp = warp_id(), lane = lane_id();
  const int ks = (int)cluster_size();
  const int rank = (int)cluster_rank();
  const bool leader = rank == 0;
  const int tile = blockIdx.x / ks;
  const int m0 = tile * kBM;
  const int kt0 = rank * k_tiles / ks, kt1 = (rank + 1) * k_tiles / ks;
  const int n_kt = kt1 - kt0;
  const uint32_t tmem_cols = leader ? G::kTmemCols : G::kL1Cols;
  QQT_PH_START(ph_t0);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_a);
    if (SPLIT_A) prefetch_tmap(&tm_alo);
    prefetch_tmap(&tm_b);
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    mbar_init(wbar, 1);
    mbar_init(abar, kEpiThreads);
    mbar_init(dbar, 1);
    mbar_init(pready, ks > 1 ? ks - 1 : 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp >= 2 && warp < 6) ktile_flags_part(TRAIN ? nullptr : tiles, m0, m0 + kBM, n_rows, kpart);
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  // every CTA's barriers are initialised before any remote arrival
  if (ks > 1) {
    cluster_arrive();
    cluster_wait();
  }
  QQT_PH_AT(1, 0, ph_t0, threadIdx.x == 0);
  QQT_PH(1, 1, threadIdx.x == 0);
  const uint32_t tmem = *tmem_slot;
  bool arrived = false;   // this thread's arrival on the closing cluster barrier
  if (test_wait) {
    // failure-path check (qqt_test_set_wait_polls): before anything is
    // issued, one bounded wait of test_wait polls on the tail-image barrier,
    // which nothing completes before layer 1 ends, expires like any wait
    // that runs out; the CTA then takes the abort path with nothing in
    // flight
    if (threadIdx.x == 0 && !mbar_wait(wbar, 0, test_wait)) *abort_flag = 1;
    __syncthreads();
  }

  if (warp == 0) {
    const uint64_t kmask = ktile_mask(kpart, k_tiles);
    // training forward over minibatch rows of a larger buffer: the tile's
    // 128 row ids (rows past the end and invalid ids read row 0; invalid ids
    // raise QQT_DEV_BAD_INDEX), fetched by TMA tile::gather4, four rows each
    int32_t* row_id = (int32_t*)(smem + G::kRegion + 256);
    const bool gather = TRAIN && tr.idx != nullptr;
    if (gather) {
      for (int i = lane; i < kBM; i += 32) {
        const int r = m0 + i;
        int64_t v = r < n_rows ? tr.idx[r] : 0;
        if (v < 0 || v >= tr.n_src) {
          flag_error(QQT_DEV_BAD_INDEX);
          v = 0;
        }
        row_id[i] = (int32_t)v;
      }
      __syncwarp();
    }
    if (lane == 0) {
      // ---------------- TMA producer (layer 1, this rank's K tiles)
      int issued_until = 0;
      // clusters start at different K tiles so that at any time they read
      // different lines of the shared weight stream from L2
      const int k0 = (int)(((unsigned)tile * 7u) % (unsigned)n_kt);
      int kt_src = kt0 + k0;
      for (int j = 0, kt = 0; j < n_kt; ++j, kt_src = kt_src + 1 == kt1 ? kt0 : kt_src + 1) {
        if (j > 0 && !ktile_in(kmask, kt_src)) continue;   // zero in every row of the tile
        const int s = kt % G::kStages;
        if (kt >= G::kStages) {
          if (!mbar_wait(&empty[s], ((kt / G::kStages) - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
        }
        if (*abort_flag) break;
        uint8_t* st = smem + s * G::kStageBytes;
        const int kx = kt_src * kBK;
        mbar_expect_tx(&full[s], G::kStageBytes);
        if (gather) {
#pragma unroll 4
          for (int g = 0; g < kBM / 4; ++g)
            tma_gather4(&tm_a, &full[s], st + g * 512, kx, row_id[4 * g], row_id[4 * g + 1],
                        row_id[4 * g + 2], row_id[4 * g + 3]);
        } else {
          tma_load_2d(&tm_a, &full[s], st, kx, m0);
        }
        if (SPLIT_A) tma_load_2d(&tm_alo, &full[s], st + G::kABytes, kx, m0);
        tma_load_2d(&tm_b, &full[s], st + G::kAAll, kx, 0);
        tma_load_2d(&tm_b, &full[s], st + G::kAAll + G::kBBytes, kx, NT);
        issued_until = ++kt;
        QQT_PH(1, 2, kt == 1);
      }
      QQT_PH(1, 3, true);
      // drain: every issued stage must land before the CTA may exit
      for (int kt = max(0, issued_until - G::kStages); kt < issued_until; ++kt)
        mbar_wait(&full[kt % G::kStages], (kt / G::kStages) & 1);
    }
  } else if (warp == 1) {
    const uint64_t kmask = ktile_mask(kpart, k_tiles);
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = idesc_f16(kBM, NT);
      const uint32_t idesc_st = idesc_f16(kBM, 256);   // one seat: hi and lo rows stacked
      // the producer's tile sequence: its length is all this loop needs
      const int n_run =
          ktile_count(kmask, kt0, kt1, kt0 + (int)(((unsigned)tile * 7u) % (unsigned)n_kt));
      bool ok = true;
      for (int kt = 0; kt < n_run && ok; ++kt) {
        const int s = kt % G::kStages;
        // an abort stops the MMAs before the next stage (the producer
        // drains every stage it issued before the CTA exits)
        if (*abort_flag || !mbar_wait(&full[s], (kt / G::kStages) & 1)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint8_t* st = smem + s * G::kStageBytes;
        const uint64_t da = sw128_desc(st);
        const uint64_t dal = sw128_desc(st + G::kABytes);
        const uint64_t dh = sw128_desc(st + G::kAAll);
        const uint64_t dl = sw128_desc(st + G::kAAll + G::kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);   // 32 bytes per K=16 step
          if (NT == 128) {
            // W_lo's rows follow W_hi's in the stage (same swizzle phase)
            umma_f16(tmem, da + off, dh + off, idesc_st, (kt > 0 || kk > 0) ? 1u : 0u);
          } else {
            umma_f16(tmem, da + off, dh + off, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
            umma_f16(tmem, da + off, dl + off, idesc, 1u);
          }
          if (SPLIT_A) umma_f16(tmem, dal + off, dh + off, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accb);   // fires once every issued MMA has completed
      QQT_PH(1, 4, true);
      if (leader) {
        // the pipeline region is free once layer 1's MMAs are done: bring in
        // the tail weight images (all CTAs read the same 160 KB, an L2 hit)
        bool loaded = false;
        if (mbar_wait(accb, 0) && ok) {
          QQT_PH(1, 5, true);
          mbar_expect_tx(wbar, kImgBytes);
          for (uint32_t o = 0; o < kImgBytes; o += 16384) bulk_load(smem + o, img + o, 16384, wbar);
          loaded = true;
        } else {
          *abort_flag = 1;
        }
        const uint32_t id2 = idesc_f16(kBM, 128), id3 = idesc_f16(kBM, 192);
        uint8_t* a_hi = smem + G::kAct;
        uint8_t* a_lo = a_hi + G::kActBytes;
        int committed = 0;
        if (loaded && !mbar_wait(wbar, 0)) *abort_flag = 1;
        QQT_PH(1, 6, true);
        for (int s = 0; s < S && !*abort_flag; ++s) {
          // layer 2: D2 overwrites this seat's layer-1 columns (already read)
          if (!mbar_wait(abar, (2 * s) & 1)) { *abort_flag = 1; break; }
          asm volatile("tcgen05.fence::after_thread_sync;");
          umma_split_k128(tmem + 128 * s, a_hi, a_lo, smem + G::kW1, smem + G::kW1 + kImgW1Bytes,
                          128, id2);
          umma_commit(dbar);
          ++committed;
          // head hidden layer
          if (!mbar_wait(abar, (2 * s + 1) & 1)) { *abort_flag = 1; break; }
          asm volatile("tcgen05.fence::after_thread_sync;");
          umma_split_k128(tmem + G::kColH, a_hi, a_lo, smem + G::kH0,
                          smem + G::kH0 + kImgH0Bytes, 192, id3);
          umma_commit(dbar);
          ++committed;
        }
        // the epilogue consumes every commit; on abort wait here for the last one
        if (*abort_flag && committed > 0) mbar_wait(dbar, (committed - 1) & 1);
        if (loaded && *abort_flag) mbar_wait(wbar, 0);
      } else {
        mbar_wait(accb, 0);   // this rank's MMAs are done before it may exit
      }
    }
  } else {
    // ---------------- epilogue: row r = 32 * (warp % 4) + lane, columns
    // 32 * quarter .. + 31 of each 128-wide layer
    const int qd = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int r = qd * 32 + lane;
    const int row = m0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    const uint32_t scr = lane_base + G::kColScr;
    uint8_t* a_hi = smem + G::kAct;
    uint8_t* a_lo = a_hi + G::kActBytes;
    // sampling inputs of this row (the thread of quarter 0 samples it)
    SampleIn sin[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
      sin[s] = SampleIn{0u, 0.f, 0.f};
      if (!TRAIN && leader && quarter == 0 && row < n_rows)
        sin[s] = sample_load(row, seat0 + s, n_rows, io.mm[s], mm_stride, io.bm[s], bm_stride, u);
    }
    bool ok = epi_and(mbar_wait(accb, 0) && *abort_flag == 0);
    QQT_PH(1, 7, warp == 2 && lane == 0);
    // layer 1 is done: a kernel launched as this one's programmatic
    // dependent (the simulator step) may start staging its state now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;");
    // this thread's 32 layer-1 sums of seat s (one seat: A W_hi + A W_lo)
    auto ld_layer1 = [&](int s, float* x) {
      if (NT == 128) {
        float y[32];
        tmem_ld32x2(lane_base + 32 * quarter, lane_base + 128 + 32 * quarter, x, y);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = __fadd_rn(x[i], y[i]);
      } else {
        tmem_ld32(lane_base + 128 * s + 32 * quarter, x);
      }
    };
    if (!leader) {
      // split-K partials -> own shared memory (the drained pipeline region)
      if (ok) {
#pragma unroll 1
        for (int s = 0; s < S; ++s) {
          float x[32];
          ld_layer1(s, x);
          uint8_t* part = smem + s * (kBM * 512);
#pragma unroll
          for (int t = 0; t < 8; ++t)
            *reinterpret_cast<float4*>(part + part_off(r, 8 * quarter + t)) =
                make_float4(x[4 * t], x[4 * t + 1], x[4 * t + 2], x[4 * t + 3]);
        }
      }
      asm volatile("fence.acq_rel.cluster;" ::: "memory");
      epi_sync();
      // one arrival per rank (also on failure: the error word is already set)
      if (warp == 2 && lane == 0) mbar_arrive_remote(dsmem_addr(pready, 0));
      // stays resident (closing cluster barrier) until rank 0 has read the partials
      cluster_arrive();
      arrived = true;
    } else {
      if (ks > 1) ok = epi_and(ok && mbar_wait_cluster(pready, 0));
#pragma unroll 1
      for (int s = 0; s < S && ok; ++s) {
        float x[32];
        // LN1 over the layer-1 pre-activations (rank-ordered split-K sum)
        ld_layer1(s, x);
#pragma unroll 1
        for (int c = 1; c < ks; ++c) {
          const uint32_t base = dsmem_addr(smem + s * (kBM * 512), (uint32_t)c);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float4 v = ld_dsmem_f4(base + part_off(r, 8 * quarter + t));
            x[4 * t] = __fadd_rn(x[4 * t], v.x);
            x[4 * t + 1] = __fadd_rn(x[4 * t + 1], v.y);
            x[4 * t + 2] = __fadd_rn(x[4 * t + 2], v.z);
            x[4 * t + 3] = __fadd_rn(x[4 * t + 3], v.w);
          }
        }
        if (ks > 1 && s == S - 1) {
          cluster_arrive();   // done reading the other ranks' shared memory
          arrived = true;
        }
        bias_ln_relu_quarter(x, quarter, scr, f + F_B0 + 128 * s, f + F_LN1G, f + F_LN1B,
                             TRAIN && row < n_rows ? tr.h1 + (size_t)row * 128 + 32 * quarter
                                                   : nullptr);
        store_split_quarter(x, a_hi, a_lo, r, quarter);
        fence_proxy_async();
        asm volatile("tcgen05.fence::before_thread_sync;");
        mbar_arrive(abar);
        QQT_PH(1, 8, warp == 2 && lane == 0);
        // LN2 over layer 2
        ok = epi_and(mbar_wait(dbar, (2 * s) & 1) && *abort_flag == 0);
        if (!ok) break;
        QQT_PH(1, 9, warp == 2 && lane == 0);
        asm volatile("tcgen05.fence::after_thread_sync;");
        tmem_ld32(lane_base + 128 * s + 32 * quarter, x);
        bias_ln_relu_quarter(x, quarter, scr + 8, f + F_B1, f + F_LN2G, f + F_LN2B,
                             TRAIN && row < n_rows ? tr.h2 + (size_t)row * 128 + 32 * quarter
                                                   : nullptr);
        store_split_quarter(x, a_hi, a_lo, r, quarter);
        fence_proxy_async();
        asm volatile("tcgen05.fence::before_thread_sync;");
        mbar_arrive(abar);
        QQT_PH(1, 10, warp == 2 && lane == 0);
        // head hidden units -> this quarter's partial output logits
        ok = epi_and(mbar_wait(dbar, (2 * s + 1) & 1) && *abort_flag == 0);
        if (!ok) break;
        QQT_PH(1, 11, warp == 2 && lane == 0);
        asm volatile("tcgen05.fence::after_thread_sync;");
        float z[8];
#pragma unroll
        for (int o = 0; o < 8; ++o) z[o] = 0.f;
        head_out_quarter(lane_base + G::kColH, quarter, f, z);
        // the four quarters' partial logits through the row's TMEM lane
        QQT_PH(1, 12, warp == 2 && lane == 0);
        tmem_st8(scr + 16 + 8 * quarter, z);
        asm volatile("tcgen05.fence::before_thread_sync;");
        quad_sync();
        asm volatile("tcgen05.fence::after_thread_sync;");
        if (quarter == 0) {
          float zz[32];
          tmem_ld32(scr + 16, zz);
          if (row < n_rows) {
#pragma unroll
            for (int o = 0; o < 8; ++o)
              z[o] = ((zz[o] + zz[8 + o]) + (zz[16 + o] + zz[24 + o])) + __ldg(f + F_HB2 + o);
            if (TRAIN)
              score_write(z, row, io.mm[s], mm_stride, io.bm[s], bm_stride, io.act[s],
                          act_stride, logp_out, tr.ent, value_out);
            else
              sample_write(z, row, seat0 + s, n_rows, sin[s], io.act[s], act_stride, logp_out,
                           value_out, logits_out);
          }
        }
      }
      if (!ok) *abort_flag = 1;
      QQT_PH(1, 13, warp == 2 && lane == 0);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  if (ks > 1) {
    if (!arrived) cluster_arrive();
    cluster_wait();
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(tmem_cols));
  }
  QQT_PH(1, 14, threadIdx.x == 0);
}

// Split-K factor for a launch of m_tiles row tiles over k_tiles K tiles:
// QQT_MLP_SPLIT_K (1..8) if set, else 4 for launches of up to 8 row tiles
// (up to 1024 envs: a small batch is latency-bound, and the split divides
// the per-SM TMA stream), 2 up to 16 tiles, and no split above that (a
// rollout's policy runs beside the simulator kernels, and extra CTAs only
// take SMs from them).
static int mlp_split_k(int m_tiles, int k_tiles) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("QQT_MLP_SPLIT_K");
    env = e ? atoi(e) : 0;
    if (env < 0 || env > kMaxSplitK) env = 0;
  }
  int ks = env;
  if (ks == 0) ks = m_tiles <= 8 ? 4 : (m_tiles <= 16 ? 2 : 1);
  return min(ks, max(1, k_tiles / 2));
}

// Poll limit of the failure-path check in k_mlp_fused; 0 (the default)
// leaves it off.  Set only by qqt_test_set_wait_polls.
static std::atomic<uint32_t> g_test_wait_polls{0};

template <int NT, bool SPLIT_A, bool TRAIN = false>
static int launch_mlp_fused(const CUtensorMap& ma, const CUtensorMap& malo, const CUtensorMap& mb,
                            int n_rows, int k_tiles, const float* f, const uint8_t* img,
                            const SeatOut& io, int seat0, int mm_stride, int bm_stride,
                            const float* u, int act_stride, float* logp, float* value,
                            float* logits, cudaStream_t st, TrainOut tr = TrainOut{},
                            const uint4* tiles = nullptr) {
  using G = FusedCfg<NT, SPLIT_A>;
  auto kern = k_mlp_fused<NT, SPLIT_A, TRAIN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  const int m_tiles = (n_rows + kBM - 1) / kBM;
  const int ks = mlp_split_k(m_tiles, k_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(m_tiles * ks), 1, 1);
  cfg.blockDim = dim3(kMlpThreads, 1, 1);
  cfg.dynamicSmemBytes = G::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ks > 1 ? 1 : 0;
  const uint32_t test_wait = g_test_wait_polls.load(std::memory_order_relaxed);
  if (cudaLaunchKernelEx(&cfg, kern, ma, malo, mb, n_rows, k_tiles, f, img, io, seat0, mm_stride,
                         bm_stride, u, act_stride, logp, value, logits, tr,
                         test_wait, tiles) != cudaSuccess)
    return QQT_E_LAUNCH;
  return launch_status();
}

}  // namespace qqt

#include "policy_pair.cu"

using namespace qqt;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// 2-D fp16 K-major tensor map: inner dim K (elements), outer dim rows.
static bool make_map(CUtensorMap* m, const void* base, uint64_t k, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static const char* kParamNames =
    "shared.0.weight shared.0.bias shared.1.weight shared.1.bias shared.3.weight shared.3.bias "
    "shared.4.weight shared.4.bias move_head.0.weight move_head.0.bias move_head.2.weight "
    "move_head.2.bias bomb_head.0.weight bomb_head.0.bias bomb_head.2.weight bomb_head.2.bias "
    "critic.0.weight critic.0.bias critic.2.weight critic.2.bias";

extern "C" const char* qqt_mlp_param_names(void) { return kParamNames; }

extern "C" uint64_t qqt_mlp_pack_bytes(int32_t k_in, int32_t n_seats) {
  if (k_in <= 0 || n_seats < 1 || n_seats > 2) return 0;
  return mlp_pack_layout(k_in, n_seats).total;
}

extern "C" int qqt_mlp_pack(const float* const* params, int32_t k_in, int32_t n_players,
                            int32_t channels, int32_t hw, int32_t n_seats, const int32_t* pids,
                            void* pack, qqt_stream_t stream) {
  if (!params || !pack || !pids || n_seats < 1 || n_seats > 2) return QQT_E_ARG;
  if (k_in != channels * hw) return QQT_E_ARG;
  if (n_players < 2 || n_players > QQT_MAX_P || channels > 64) return QQT_E_ARG;
  for (int i = 0; i < 20; ++i)
    if (!params[i]) return QQT_E_ARG;
  const MlpPack L = mlp_pack_layout(k_in, n_seats);
  // source channel of each stored channel for each seat: inverse of the view permutation
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
    // view channel v reads stored channel perm[v]; W0's column block v pairs with
    // view channel v, so stored channel perm[v] takes W0 block v
    for (int v = 0; v < channels; ++v) sc.src[s][perm[v]] = v;
  }
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* pk = (uint8_t*)pack;
  const size_t total = (size_t)L.nt * L.kp;
  k_mlp_pack_w0<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      params[0], k_in, L.kp, hw, channels, sc, L.nt, (__half*)(pk + L.b_off));
  HeadParams hp;
  hp.b0 = params[1];
  hp.ln1g = params[2];
  hp.ln1b = params[3];
  hp.w1 = params[4];
  hp.b1 = params[5];
  hp.ln2g = params[6];
  hp.ln2b = params[7];
  hp.mw0 = params[8];
  hp.mb0 = params[9];
  hp.mw2 = params[10];
  hp.mb2 = params[11];
  hp.bw0 = params[12];
  hp.bb0 = params[13];
  hp.bw2 = params[14];
  hp.bb2 = params[15];
  hp.cw0 = params[16];
  hp.cb0 = params[17];
  hp.cw2 = params[18];
  hp.cb2 = params[19];
  k_mlp_pack_rest<<<(128 * 128 + 255) / 256, 256, 0, st>>>(hp, n_seats, (float*)(pk + L.f_off));
  k_mlp_pack_images<<<(192 * 128 + 255) / 256, 256, 0, st>>>(hp, pk + L.img_off);
  k_mlp_pack_pair_images<<<(192 * 128 + 255) / 256, 256, 0, st>>>(hp, pk + L.pair_off);
  return launch_status();
}

// The fused kernel keeps every intermediate on chip; `work` is reserved.
extern "C" uint64_t qqt_mlp_work_bytes(int32_t n_envs, int32_t n_seats) {
  (void)n_envs;
  (void)n_seats;
  return 256;
}

extern "C" int qqt_mlp_act(const void* pack, const void* obs, const uint32_t* obs_tiles,
                           int32_t n_envs, int32_t obs_stride,
                           int32_t k_in, int32_t n_seats, const uint8_t* const* mm,
                           int32_t mm_stride, const uint8_t* const* bm, int32_t bm_stride,
                           const float* u, int64_t* const* act, int32_t act_stride, float* logp,
                           float* value, float* logits, void* work, qqt_stream_t stream) {
  (void)work;
  if (!pack || !obs || !mm || !bm || !u || !act) return QQT_E_ARG;
  if (n_envs <= 0 || n_seats < 1 || n_seats > 2 || mm_stride < 5 || bm_stride < 2 ||
      act_stride < 2)
    return QQT_E_ARG;
  for (int s = 0; s < n_seats; ++s)
    if (!mm[s] || !bm[s] || !act[s]) return QQT_E_ARG;
  if (obs_stride % 8 || obs_stride < k_in || ((uintptr_t)obs & 15) || ((uintptr_t)pack & 255) ||
      ((uintptr_t)obs_tiles & 15))
    return QQT_E_ALIGN;
  const uint4* tiles = reinterpret_cast<const uint4*>(obs_tiles);
  const MlpPack L = mlp_pack_layout(k_in, n_seats);
  const uint8_t* pk = (const uint8_t*)pack;
  CUtensorMap ma, mb;
  if (!make_map(&ma, obs, (uint64_t)obs_stride, (uint64_t)n_envs, (uint64_t)obs_stride * 2, kBM))
    return QQT_E_ARG;
  if (!make_map(&mb, pk + L.b_off, (uint64_t)L.kp, (uint64_t)2 * L.nt, (uint64_t)L.kp * 2,
                (uint32_t)L.nt))
    return QQT_E_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const float* fpar = (const float*)(pk + L.f_off);
  const int k_tiles = L.kp / kBK;
  SeatOut io;
  for (int s = 0; s < 2; ++s) {
    io.mm[s] = s < n_seats ? mm[s] : nullptr;
    io.bm[s] = s < n_seats ? bm[s] : nullptr;
    io.act[s] = s < n_seats ? act[s] : nullptr;
  }
  const int m_tiles = (n_envs + kBM - 1) / kBM;
  if (L.nt == 256 && mlp_pair_enabled() && mlp_split_k(m_tiles, k_tiles) == 1) {
    // large two-seat batch: SM pairs, each CTA streaming half of the weights
    CUtensorMap mbh;
    if (!make_map(&mbh, pk + L.b_off, (uint64_t)L.kp, (uint64_t)2 * L.nt, (uint64_t)L.kp * 2,
                  (uint32_t)(L.nt / 2)))
      return QQT_E_ARG;
    return launch_mlp_pair<256>(ma, mbh, n_envs, k_tiles, fpar, pk + L.pair_off, io, mm_stride,
                                bm_stride, u, act_stride, logp, value, logits, st, tiles);
  }
  if (L.nt == 128)
    return launch_mlp_fused<128, false>(ma, ma, mb, n_envs, k_tiles, fpar, pk + L.img_off, io, 0,
                                        mm_stride, bm_stride, u, act_stride, logp, value, logits,
                                        st, TrainOut{}, tiles);
  return launch_mlp_fused<256, false>(ma, ma, mb, n_envs, k_tiles, fpar, pk + L.img_off, io, 0,
                                      mm_stride, bm_stride, u, act_stride, logp, value, logits, st,
                                      TrainOut{}, tiles);
}

extern "C" int qqt_test_set_wait_polls(uint32_t polls) {
  g_test_wait_polls.store(polls, std::memory_order_relaxed);
  return QQT_OK;
}
