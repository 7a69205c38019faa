// First layer of the MLP policy's PPO update on the 5th-generation tensor
// cores (train/ppo.py:364-437 through ActorCritic(mlp), train/model.py:121-153).
//
// Every minibatch of the reference's update runs Linear(2366 -> 128) in
// float32 twice: the forward product over the minibatch's observation rows
// (an index gather, then a float16 -> float32 copy, then an fp32 GEMM) and
// autograd's weight gradient, a second fp32 GEMM with the minibatch as its
// reduction axis.  These kernels do the same arithmetic from the float16 rows
// themselves:
//
// k_gather_rows   the minibatch's rows of the rollout's fp16 observation
//                 buffer into one contiguous block: one warp per row, 16-byte
//                 copies, every index checked against the buffer's row count.
// k_l1_fwd        h1 = x W0p^T + b0 (W0p = W0 with the seat's view
//                 permutation folded into its column order, stored as fp16 hi
//                 and lo halves by k_mlp_pack_w0): persistent CTAs over
//                 128-row tiles.  Warp 0 streams the K tiles of x and W0p with
//                 TMA (no multicast), warp 1 issues tcgen05.mma kind::f16
//                 (x*Whi + x*Wlo, fp32 accumulate) into one of two TMEM
//                 accumulators while warps 2-5 drain the other (bias add,
//                 float32 rows out).  x is exact in fp16, so the products
//                 carry W0's float32 precision.
// k_absmax, k_dh_split
//                 dL/dh1 times a power of two that puts its largest magnitude
//                 just under 2^14, split into fp16 hi and lo halves: 22
//                 significant bits of every value, and no value leaves fp16's
//                 range.
// k_l1_wgrad      G = dh1^T x over the minibatch: M = 128 hidden units, N = 256
//                 observation columns per CTA (64 in the last block), K = the
//                 CTA's slice of rows.  Both operands are read in their stored
//                 row order, so both are MN-major: 128-byte swizzle atoms of
//                 64 elements x 8 rows, atoms 1024 bytes apart along K and
//                 64-element blocks one TMA box apart along M / N.  Two MMAs
//                 per K step (dh_hi*x + dh_lo*x).  Each CTA writes its fp32
//                 partial sums to the workspace.
// k_wgrad_reduce  dW0 = (sum of the K slices in slice order) / scale, stored in
//                 W0's own column order (the inverse of the view permutation).
//
// Every mbarrier wait is bounded (mbar_wait); on expiry the CTA raises
// QQT_DEV_TIMEOUT, waits (bounded) for the copies and MMAs it issued, frees
// its TMEM and returns.

namespace qqt {

// ---------------------------------------------------------------- gather

__global__ void k_gather_rows(const uint4* __restrict__ src, int64_t src_stride16, int64_t n_src,
                              const int64_t* __restrict__ idx, int64_t n,
                              uint4* __restrict__ dst, int64_t dst_stride16, int row16) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = lane_id();
  if (w >= n) return;
  const int64_t r = __ldg(idx + w);
  uint4* d = dst + w * dst_stride16;
  if (r < 0 || r >= n_src) {
    if (lane == 0) flag_error(QQT_DEV_BAD_INDEX);
    for (int c = lane; c < row16; c += 32) d[c] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* s = src + r * src_stride16;
#pragma unroll 4
  for (int c = lane; c < row16; c += 32) d[c] = __ldcs(s + c);
}

// ---------------------------------------------------------------- forward

constexpr int kL1Stages = 4;
constexpr int kL1Tile = kBM * kBK * 2;                  // 16 KB: x tile or one W half
constexpr int kL1StageBytes = 3 * kL1Tile;
constexpr int kL1Threads = 192;                         // producer, MMA, 4 epilogue warps
constexpr int kL1Smem = kL1Stages * kL1StageBytes + 1024 + 256;
static_assert(kL1Smem <= 232448, "layer-1 forward shared memory");

__global__ void __launch_bounds__(kL1Threads, 1)
k_l1_fwd(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
         int n_rows, int k_tiles, const float* __restrict__ b0, float* __restrict__ h1) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + kL1Stages * kL1StageBytes);
  uint64_t* empty = full + kL1Stages;
  uint64_t* tfull = empty + kL1Stages;    // [2] accumulator b complete
  uint64_t* tempty = tfull + 2;           // [2] accumulator b drained (128 arrivals)
  uint64_t* done = tempty + 2;            // every issued MMA complete
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  const int n_tiles = (n_rows + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kL1Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % kL1Stages;
          if (it >= kL1Stages && !mbar_wait(&empty[s], ((it / kL1Stages) - 1) & 1)) {
            ok = false;
            break;
          }
          if (*abort_flag) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kL1StageBytes;
          mbar_expect_tx(&full[s], kL1StageBytes);
          tma_load_2d(&tm_x, &full[s], st, kt * kBK, tile * kBM);
          tma_load_2d(&tm_w, &full[s], st + kL1Tile, kt * kBK, 0);
          tma_load_2d(&tm_w, &full[s], st + 2 * kL1Tile, kt * kBK, kBM);
        }
      }
      if (!ok) *abort_flag = 1;
      // drain: every issued stage lands before the CTA may exit
      for (int j = max(0, it - kL1Stages); j < it; ++j)
        mbar_wait(&full[j % kL1Stages], (j / kL1Stages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = idesc_f16(kBM, 128);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++lt) {
        const int b = lt & 1;
        if (lt >= 2 && !mbar_wait(&tempty[b], ((lt >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t d = tmem + 128u * (uint32_t)b;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % kL1Stages;
          if (!mbar_wait(&full[s], (it / kL1Stages) & 1) || *abort_flag) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;");
          uint8_t* st = smem + s * kL1StageBytes;
          const uint64_t da = sw128_desc(st);
          const uint64_t dh = sw128_desc(st + kL1Tile);
          const uint64_t dl = sw128_desc(st + 2 * kL1Tile);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t off = (uint64_t)((kk * 32) >> 4);   // 32 bytes per K=16 step
            umma_f16(d, da + off, dh + off, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
            umma_f16(d, da + off, dl + off, idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(done);
      mbar_wait(done, 0);
    }
  } else {
    // ---------------- epilogue: warp w drains TMEM lanes 32*(w%4) .. +31
    const int qd = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    int lt = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (lt >> 1) & 1) && !*abort_flag);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;");
      const int r = tile * kBM + qd * 32 + lane;
      float4* out = reinterpret_cast<float4*>(h1 + (size_t)r * 128);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(lane_base + 128u * (uint32_t)b + 32u * (uint32_t)c, v);
        if (c == 3) {
          asm volatile("tcgen05.fence::before_thread_sync;");
          mbar_arrive(&tempty[b]);
        }
        if (r < n_rows) {
          const float4* bias = reinterpret_cast<const float4*>(b0 + 32 * c);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bv = __ldg(bias + i);
            out[8 * c + i] = make_float4(v[4 * i] + bv.x, v[4 * i + 1] + bv.y,
                                         v[4 * i + 2] + bv.z, v[4 * i + 3] + bv.w);
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

// ---------------------------------------------------------------- dL/dh1 split

// Exponent s of the power-of-two scale 2^s applied to dL/dh1: the largest
// magnitude a lands in [2^13, 2^14).  |s| <= 100 keeps 2^s and 2^-s normal
// floats; a zero or non-finite maximum gives s = 0.
__device__ __forceinline__ int dh_scale_exp(const uint32_t* amax_bits) {
  const uint32_t bits = *amax_bits;
  const int E = (int)((bits >> 23) & 0xFF);
  if (bits == 0u || E == 0xFF) return 0;
  const int e = (E == 0 ? -126 : E - 126);   // a = m * 2^e, m in [0.5, 1)
  return max(-100, min(100, 14 - e));
}

__device__ __forceinline__ float pow2f(int s) { return __int_as_float((127 + s) << 23); }

__global__ void k_absmax(const float4* __restrict__ x, int64_t n4, uint32_t* __restrict__ out) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(x + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  // non-negative floats order like their bit patterns
  const uint32_t w = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
  if (lane_id() == 0 && w != 0u) atomicMax(out, w);
}

__global__ void k_dh_split(const float4* __restrict__ dh, int64_t n4,
                           const uint32_t* __restrict__ amax_bits, uint2* __restrict__ hi,
                           uint2* __restrict__ lo) {
  const float scale = pow2f(dh_scale_exp(amax_bits));
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(dh + i);
    const float a[4] = {v.x * scale, v.y * scale, v.z * scale, v.w * scale};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __float2half_rn(a[j]);
      l[j] = __float2half_rn(a[j] - __half2float(h[j]));
    }
    uint2 ph, pl;
    ph.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
    ph.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
    pl.x = (uint32_t)__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[1]) << 16);
    pl.y = (uint32_t)__half_as_ushort(l[2]) | ((uint32_t)__half_as_ushort(l[3]) << 16);
    hi[i] = ph;
    lo[i] = pl;
  }
}

// ---------------------------------------------------------------- weight gradient

constexpr int kWgStages = 3;
constexpr int kWgBK = 64;                                 // minibatch rows per stage
constexpr int kWgBox = 64 * 64 * 2;                       // 8 KB: 64 rows x 64 columns
constexpr int kWgA = 2 * kWgBox;                          // 128 hidden units (hi or lo)
constexpr int kWgN = 256;                                 // observation columns per CTA
constexpr int kWgStageBytes = 2 * kWgA + (kWgN / 64) * kWgBox;   // 64 KB
constexpr int kWgThreads = 192;
constexpr int kWgSmem = kWgStages * kWgStageBytes + 1024 + 256;
static_assert(kWgSmem <= 232448, "weight-gradient shared memory");

// MN-major operand tile with the 128-byte swizzle: rows of 64 elements (128
// bytes) along M / N, 8-row atoms 1024 bytes apart along K (stride byte
// offset), 64-element blocks `lbo` bytes apart (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mn_desc(const void* tile, uint32_t lbo) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: fp16 A/B, fp32 D, both operands MN-major.
__host__ __device__ constexpr uint32_t idesc_f16_mn(int m, int n) {
  return (1u << 4) | (1u << 15) | (1u << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__global__ void __launch_bounds__(kWgThreads, 1)
k_l1_wgrad(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
           const __grid_constant__ CUtensorMap tm_x, int n_rows, int kp, float* __restrict__ part) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + kWgStages * kWgStageBytes);
  uint64_t* empty = full + kWgStages;
  uint64_t* accb = empty + kWgStages;
  uint32_t* tmem_slot = (uint32_t*)(accb + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  const int n0 = blockIdx.x * kWgN;
  const int nw = min(kWgN, kp - n0);                      // a multiple of 64
  const int n_blk = nw / 64;
  const int k_st = (n_rows + kWgBK - 1) / kWgBK;
  const int s0 = (int)((int64_t)blockIdx.y * k_st / gridDim.y);
  const int s1 = (int)((int64_t)(blockIdx.y + 1) * k_st / gridDim.y);
  const int n_st = s1 - s0;
  const uint32_t stage_tx = (uint32_t)(2 * kWgA + n_blk * kWgBox);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_st; ++i) {
        const int s = i % kWgStages;
        if (i >= kWgStages && !mbar_wait(&empty[s], ((i / kWgStages) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = smem + s * kWgStageBytes;
        const int y = (s0 + i) * kWgBK;
        mbar_expect_tx(&full[s], stage_tx);
        tma_load_2d(&tm_hi, &full[s], st, 0, y);
        tma_load_2d(&tm_hi, &full[s], st + kWgBox, 64, y);
        tma_load_2d(&tm_lo, &full[s], st + kWgA, 0, y);
        tma_load_2d(&tm_lo, &full[s], st + kWgA + kWgBox, 64, y);
        for (int q = 0; q < n_blk; ++q)
          tma_load_2d(&tm_x, &full[s], st + 2 * kWgA + q * kWgBox, n0 + 64 * q, y);
        issued = i + 1;
      }
      for (int j = max(0, issued - kWgStages); j < issued; ++j)
        mbar_wait(&full[j % kWgStages], (j / kWgStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_mn(128, nw);
      for (int i = 0; i < n_st; ++i) {
        const int s = i % kWgStages;
        if (!mbar_wait(&full[s], (i / kWgStages) & 1) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint8_t* st = smem + s * kWgStageBytes;
        const uint64_t dah = sw128_mn_desc(st, kWgBox);
        const uint64_t dal = sw128_mn_desc(st + kWgA, kWgBox);
        const uint64_t db = sw128_mn_desc(st + 2 * kWgA, kWgBox);
#pragma unroll
        for (int kk = 0; kk < kWgBK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 2048) >> 4);   // two 8-row atoms per K=16
          umma_f16(tmem, dah + off, db + off, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tmem, dal + off, db + off, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accb);
      mbar_wait(accb, 0);
    }
  } else {
    // ---------------- epilogue: hidden unit j = TMEM lane, nw columns
    const int qd = warp & 3;
    const int j = qd * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accb, 0) && !*abort_flag);
    asm volatile("tcgen05.fence::after_thread_sync;");
    float4* out = reinterpret_cast<float4*>(part + ((size_t)blockIdx.y * 128 + j) * kp + n0);
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < n_blk * 2; ++c) {
        float v[32];
        tmem_ld32(lane_base + 32u * (uint32_t)c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool z = n_st == 0;   // no MMA ran: the accumulator was never written
          out[8 * c + i] = z ? make_float4(0.f, 0.f, 0.f, 0.f)
                             : make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

struct ColumnSource {
  int32_t block[64];   // W0 column block of stored channel c
};

__global__ void k_wgrad_reduce(const float* __restrict__ part, int k_slices, int kp, int k_in,
                               int hw, ColumnSource cs, const uint32_t* __restrict__ amax_bits,
                               float* __restrict__ dw0) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)128 * k_in) return;
  const int j = (int)(i / k_in), c = (int)(i - (int64_t)j * k_in);
  float s = 0.f;
  for (int k = 0; k < k_slices; ++k) s += __ldg(part + ((size_t)k * 128 + j) * kp + c);
  const int ch = c / hw, cell = c - ch * hw;
  dw0[(size_t)j * k_in + cs.block[ch] * hw + cell] = s * pow2f(-dh_scale_exp(amax_bits));
}

// ---------------------------------------------------------------- host side

// Stored channel -> W0 column block for seat `pid` (the inverse of
// sim/config.py view_perm: view channel v reads stored channel perm[v] and
// pairs with W0's column block v).
static bool seat_column_blocks(int n_players, int channels, int pid, int32_t* block) {
  if (n_players < 2 || n_players > QQT_MAX_P || channels > 64 || pid < 0 || pid >= n_players)
    return false;
  const int base = 2 * n_players + 3;
  if (channels < base) return false;
  int perm[64], j = 0;
  perm[j++] = pid;
  perm[j++] = n_players + pid;
  for (int i = 0; i < n_players; ++i)
    if (i != pid) perm[j++] = i;
  for (int i = 0; i < n_players; ++i)
    if (i != pid) perm[j++] = n_players + i;
  perm[j++] = 2 * n_players;
  perm[j++] = 2 * n_players + 1;
  perm[j++] = 2 * n_players + 2;
  for (int c = base; c < channels; ++c) perm[j++] = c;
  for (int v = 0; v < channels; ++v) block[perm[v]] = v;
  return true;
}

static int wgrad_slices(int n_rows, int kp) {
  const int n_blocks = (kp + kWgN - 1) / kWgN;
  const int k_st = (n_rows + kWgBK - 1) / kWgBK;
  return max(1, min(sm_count() / n_blocks, k_st));
}

struct WgradWork {
  size_t amax, hi, lo, part, total;
};

static WgradWork wgrad_work_layout(int64_t n_rows, int kp) {
  WgradWork w;
  const size_t dh_bytes = ((size_t)n_rows * 128 * 2 + 1023) / 1024 * 1024;
  w.amax = 0;
  w.hi = 1024;
  w.lo = w.hi + dh_bytes;
  w.part = w.lo + dh_bytes;
  w.total = w.part + (size_t)wgrad_slices((int)n_rows, kp) * 128 * kp * 4;
  return w;
}

}  // namespace qqt

extern "C" uint64_t qqt_l1_pack_bytes(int32_t k_in) {
  if (k_in <= 0) return 0;
  const int kp = (k_in + kBK - 1) / kBK * kBK;
  return (uint64_t)2 * 128 * kp * 2;
}

extern "C" int qqt_l1_pack(const float* w0, int32_t k_in, int32_t n_players, int32_t channels,
                           int32_t hw, int32_t pid, void* pack, qqt_stream_t stream) {
  if (!w0 || !pack || k_in <= 0 || k_in != channels * hw) return QQT_E_ARG;
  if ((uintptr_t)pack & 255) return QQT_E_ALIGN;
  SeatChannels sc;
  memset(&sc, 0, sizeof(sc));
  if (!seat_column_blocks(n_players, channels, pid, sc.src[0])) return QQT_E_ARG;
  const int kp = (k_in + kBK - 1) / kBK * kBK;
  const size_t total = (size_t)128 * kp;
  k_mlp_pack_w0<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      w0, k_in, kp, hw, channels, sc, 128, (__half*)pack);
  return launch_status();
}

extern "C" int qqt_gather_rows(const void* src, int64_t n_src, int64_t src_stride_bytes,
                               const int64_t* idx, int64_t n, void* dst,
                               int64_t dst_stride_bytes, int64_t row_bytes, qqt_stream_t stream) {
  if (!src || !idx || !dst || n < 0 || n_src <= 0 || row_bytes <= 0) return QQT_E_ARG;
  if (((uintptr_t)src | (uintptr_t)dst | (uintptr_t)src_stride_bytes |
       (uintptr_t)dst_stride_bytes | (uintptr_t)row_bytes) & 15)
    return QQT_E_ALIGN;
  if (row_bytes > src_stride_bytes || row_bytes > dst_stride_bytes) return QQT_E_ARG;
  if (n == 0) return QQT_OK;
  const int64_t threads = n * 32;
  k_gather_rows<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)src, src_stride_bytes / 16, n_src, idx, n, (uint4*)dst, dst_stride_bytes / 16,
      (int)(row_bytes / 16));
  return launch_status();
}

extern "C" int qqt_l1_forward(const void* pack, const void* x, int64_t n_rows, int32_t x_stride,
                              int32_t k_in, const float* b0, float* h1, qqt_stream_t stream) {
  if (!pack || !x || !b0 || !h1 || n_rows <= 0 || k_in <= 0 || x_stride < k_in) return QQT_E_ARG;
  if (n_rows > (int64_t)0x7fffff00) return QQT_E_LIMIT;
  if ((x_stride % 8) || ((uintptr_t)x & 15) || ((uintptr_t)pack & 255) || ((uintptr_t)h1 & 15) ||
      ((uintptr_t)b0 & 15))
    return QQT_E_ALIGN;
  const int kp = (k_in + kBK - 1) / kBK * kBK;
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, (uint64_t)k_in, (uint64_t)n_rows, (uint64_t)x_stride * 2, kBM))
    return QQT_E_ARG;
  if (!make_map(&mw, pack, (uint64_t)kp, 256, (uint64_t)kp * 2, kBM)) return QQT_E_ARG;
  cudaFuncSetAttribute(k_l1_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, kL1Smem);
  const int n_tiles = (int)((n_rows + kBM - 1) / kBM);
  const int grid = min(n_tiles, sm_count());
  k_l1_fwd<<<grid, kL1Threads, kL1Smem, (cudaStream_t)stream>>>(mx, mw, (int)n_rows, kp / kBK,
                                                                 b0, h1);
  return launch_status();
}

extern "C" uint64_t qqt_l1_wgrad_work_bytes(int64_t n_rows, int32_t k_in) {
  if (n_rows <= 0 || k_in <= 0) return 0;
  const int kp = (k_in + kBK - 1) / kBK * kBK;
  return wgrad_work_layout(n_rows, kp).total;
}

extern "C" int qqt_l1_wgrad(const void* x, int64_t n_rows, int32_t x_stride, int32_t k_in,
                            const float* dh1, int32_t n_players, int32_t channels, int32_t hw,
                            int32_t pid, float* dw0, void* work, qqt_stream_t stream) {
  if (!x || !dh1 || !dw0 || !work || n_rows <= 0 || k_in <= 0 || x_stride < k_in ||
      k_in != channels * hw)
    return QQT_E_ARG;
  if (n_rows > (int64_t)0x7fffff00) return QQT_E_LIMIT;
  if ((x_stride % 8) || ((uintptr_t)x & 15) || ((uintptr_t)dh1 & 15) || ((uintptr_t)work & 1023))
    return QQT_E_ALIGN;
  ColumnSource cs;
  memset(&cs, 0, sizeof(cs));
  if (!seat_column_blocks(n_players, channels, pid, cs.block)) return QQT_E_ARG;
  const int kp = (k_in + kBK - 1) / kBK * kBK;
  const WgradWork L = wgrad_work_layout(n_rows, kp);
  uint8_t* wk = (uint8_t*)work;
  uint32_t* amax = (uint32_t*)(wk + L.amax);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(amax, 0, 4, st) != cudaSuccess) return QQT_E_LAUNCH;
  const int64_t n4 = n_rows * 32;
  const int sms = sm_count();
  const unsigned g4 = (unsigned)max((int64_t)1, min((n4 + 255) / 256, (int64_t)sms * 8));
  k_absmax<<<g4, 256, 0, st>>>((const float4*)dh1, n4, amax);
  k_dh_split<<<g4, 256, 0, st>>>((const float4*)dh1, n4, amax, (uint2*)(wk + L.hi),
                                 (uint2*)(wk + L.lo));
  CUtensorMap mh, ml, mx;
  if (!make_map(&mh, wk + L.hi, 128, (uint64_t)n_rows, 256, kWgBK) ||
      !make_map(&ml, wk + L.lo, 128, (uint64_t)n_rows, 256, kWgBK) ||
      !make_map(&mx, x, (uint64_t)k_in, (uint64_t)n_rows, (uint64_t)x_stride * 2, kWgBK))
    return QQT_E_ARG;
  cudaFuncSetAttribute(k_l1_wgrad, cudaFuncAttributeMaxDynamicSharedMemorySize, kWgSmem);
  const int slices = wgrad_slices((int)n_rows, kp);
  const dim3 grid((unsigned)((kp + kWgN - 1) / kWgN), (unsigned)slices);
  float* part = (float*)(wk + L.part);
  k_l1_wgrad<<<grid, kWgThreads, kWgSmem, st>>>(mh, ml, mx, (int)n_rows, kp, part);
  const int64_t n_out = (int64_t)128 * k_in;
  k_wgrad_reduce<<<(unsigned)((n_out + 255) / 256), 256, 0, st>>>(part, slices, kp, k_in, hw, cs,
                                                                 amax, dw0);
  return launch_status();
}
