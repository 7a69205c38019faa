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
//                 buffer (and of the packed per-row side data) into one
//                 contiguous block: a warp per observation row, several small
//                 rows per warp, 16-byte copies, every index checked against
//                 the buffer's row count.
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

// `lanes` lanes (a power of two dividing 32) copy one row, so a warp moves
// 32 / lanes rows of up to lanes x 16 bytes at once (small side-data rows
// as well as 4.7 KB observation rows, which take the whole warp).
__global__ void k_gather_rows(const uint4* __restrict__ src, int64_t src_stride16, int64_t n_src,
                              const int64_t* __restrict__ idx, int64_t n,
                              uint4* __restrict__ dst, int64_t dst_stride16, int row16,
                              int lanes) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = lane_id();
  const int l = lane & (lanes - 1);
  const int64_t w = (t >> 5) * (32 / lanes) + lane / lanes;
  if (w >= n) return;
  const int64_t r = __ldg(idx + w);
  uint4* d = dst + w * dst_stride16;
  if (r < 0 || r >= n_src) {
    if (l == 0) flag_error(QQT_DEV_BAD_INDEX);
    for (int c = l; c < row16; c += lanes) d[c] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* s = src + r * src_stride16;
#pragma unroll 4
  for (int c = l; c < row16; c += lanes) d[c] = __ldcs(s + c);
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

__global__ void k_absmax_n(const float* __restrict__ x, int64_t n, uint32_t* __restrict__ out) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__ldg(x + i)));
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
constexpr int kWgSmem = kWgStages * kWgStageBytes + 1024 + 256 + 256 /*row ids*/;
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
           const __grid_constant__ CUtensorMap tm_x, int n_rows, int kp, float* __restrict__ part,
           const int64_t* __restrict__ idx, int n_src) {
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
    // the whole warp stages a minibatch's row ids (gathered x rows: row r of
    // the minibatch is row idx[r] of the x map; rows past the end and
    // invalid ids read row 0, invalid ids raise QQT_DEV_BAD_INDEX); lane 0
    // waits on the barriers and issues the copies
    int32_t* row_id = (int32_t*)(smem + kWgStages * kWgStageBytes + 256);
    const bool gather = idx != nullptr;
    int issued = 0;
    for (int i = 0; i < n_st; ++i) {
      const int s = i % kWgStages;
      const int y = (s0 + i) * kWgBK;
      bool go = true;
      if (lane == 0) {
        if (i >= kWgStages && !mbar_wait(&empty[s], ((i / kWgStages) - 1) & 1)) {
          *abort_flag = 1;
          go = false;
        }
        if (*abort_flag) go = false;
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (gather) {
        for (int j = lane; j < kWgBK; j += 32) {
          const int r = y + j;
          int64_t v = r < n_rows ? idx[r] : 0;
          if (v < 0 || v >= n_src) {
            flag_error(QQT_DEV_BAD_INDEX);
            v = 0;
          }
          row_id[j] = (int32_t)v;
        }
        __syncwarp();
      }
      if (lane == 0) {
        uint8_t* st = smem + s * kWgStageBytes;
        mbar_expect_tx(&full[s], stage_tx);
        tma_load_2d(&tm_hi, &full[s], st, 0, y);
        tma_load_2d(&tm_hi, &full[s], st + kWgBox, 64, y);
        tma_load_2d(&tm_lo, &full[s], st + kWgA, 0, y);
        tma_load_2d(&tm_lo, &full[s], st + kWgA + kWgBox, 64, y);
        for (int q = 0; q < n_blk; ++q) {
          uint8_t* dst = st + 2 * kWgA + q * kWgBox;
          if (gather) {
            for (int g = 0; g < kWgBK / 4; ++g)
              tma_gather4(&tm_x, &full[s], dst + g * 512, n0 + 64 * q, row_id[4 * g],
                          row_id[4 * g + 1], row_id[4 * g + 2], row_id[4 * g + 3]);
          } else {
            tma_load_2d(&tm_x, &full[s], dst, n0 + 64 * q, y);
          }
        }
        issued = i + 1;
      }
      __syncwarp();   // lane 0 has read this stage's row ids before they are replaced
    }
    if (lane == 0)
      for (int j = max(0, issued - kWgStages); j < issued; ++j)
        mbar_wait(&full[j % kWgStages], (j / kWgStages) & 1);
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

// ---------------------------------------------------------------- tail backward
//
// The layers above the first, backward, for every row of a minibatch
// (train/model.py:121-153 through autograd).  Two persistent kernels with
// the block layout of k_mlp_fused (warp 0 loads, warp 1 issues MMAs, 16
// epilogue warps with four threads per row: TMEM lane quadrant x column
// quarter):
//
// k_tail_heads_bwd  per 128-row tile: LN2 of the saved h2 -> r2 (the same
//   operations as the forward, so the values agree bit for bit) -> fp16 hi/lo
//   operand; u = r2 Wh0^T on the tensor cores (the three head hidden layers,
//   N = 192); per row the head outputs, the masked log-softmax of each head
//   and, from the incoming dL/dlogp, dL/dentropy, dL/dvalue, the gradient of
//   every logit; back through the output layers and the ReLUs to dL/du,
//   scaled by a power of two bounded from the incoming gradients and split
//   into fp16 hi / lo.  Then dr2 = du Wh0 (Wh0's operand image read MN-major)
//   and dWh0^T += r2^T du (both operands MN-major views of the K-major
//   images), accumulated in TMEM over all the CTA's tiles; LN2 backward to
//   dL/dh2 (written out, float32).
// k_tail_trunk_bwd  per tile: LN1 of the saved h1 -> r1 operand; dL/dh2
//   scaled by the power of two from its maximum -> hi/lo operand;
//   dr1 = dh2 W1 and dW1^T += r1^T dh2 in TMEM; LN1 backward to dL/dh1.
//
// Small gradients (biases, LayerNorm affine, the head output layers) are
// summed over each warp's 32 rows by a shuffle reduce-scatter (lane l keeps
// element l of a 32-vector) into per-thread registers; the per-CTA partial
// sums are combined in a fixed order by k_tail_reduce.

constexpr uint32_t kTbScr = 384;                   // TMEM row-exchange scratch columns
constexpr uint32_t kTbAcc = 432;                   // heads kernel: per-thread sums (4 x 9)
constexpr int kActB = kBM * 128 * 2;               // one fp16 [128 x 128] operand image
constexpr int kThWh = 0;                           // heads kernel: Wh0 image hi, lo
constexpr int kThR = 2 * (int)kImgH0Bytes;         //   r2 operand hi, lo
constexpr int kThD = kThR + 2 * kActB;             //   du operand hi, lo (two heads at a time)
constexpr int kThBytes = kThD + 2 * kActB;
constexpr int kThSmem = kThBytes + 1024 + 256;
constexpr int kTtW = 0;                            // trunk kernel: W1 image hi, lo
constexpr int kTtR = 2 * (int)kImgW1Bytes;         //   r1 operand hi, lo
constexpr int kTtD = kTtR + 2 * kActB;             //   dh2 operand hi, lo
constexpr int kTtBytes = kTtD + 2 * kActB;
constexpr int kTtSmem = kTtBytes + 1024 + 256;
constexpr int kThAcc = 9;                          // per-thread small-gradient accumulators
constexpr int kTtAcc = 3;
static_assert(kThSmem <= 232448 && kTtSmem <= 232448, "tail backward shared memory");

__device__ __forceinline__ void tmem_st2(uint32_t taddr, float a, float b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr),
               "r"(__float_as_uint(a)), "r"(__float_as_uint(b))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}


// TMEM column += v (this thread's lane).
__device__ __forceinline__ void tmem_acc(uint32_t col, float v) {
  float o[4];
  tmem_ld4(col, o);
  tmem_st1(col, o[0] + v);
}

// Sum of a[32] over the warp's 32 lanes, element `lane` kept by each lane
// (five halving exchanges; a is clobbered).
__device__ __forceinline__ float reduce_scatter32(float* a) {
  const int lane = lane_id();
#pragma unroll
  for (int st = 0; st < 5; ++st) {
    const int s = 16 >> st;
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < (16 >> st); ++i) {
      const float send = up ? a[i] : a[i + (16 >> st)];
      const float keep = up ? a[i + (16 >> st)] : a[i];
      a[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return a[0];
}

// Mean and 1/sqrt(var + 1e-5) of the row (this thread holds 32 of its 128
// values) in bias_ln_relu_quarter's operation order.
__device__ __forceinline__ void ln_stats_quarter(const float* x, int q, uint32_t scr, float& mean,
                                                 float& rstd) {
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; i += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) s4[j] += x[i + j];
  float p[4];
  row_exchange4(scr, q, (s4[0] + s4[1]) + (s4[2] + s4[3]), p);
  mean = ((p[0] + p[1]) + (p[2] + p[3])) * (1.f / 128.f);
  float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; i += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = x[i + j] - mean;
      v4[j] = fmaf(d, d, v4[j]);
    }
  row_exchange4(scr + 4, q, (v4[0] + v4[1]) + (v4[2] + v4[3]), p);
  rstd = rsqrtf(((p[0] + p[1]) + (p[2] + p[3])) * (1.f / 128.f) + 1e-5f);
}

// 32 floats of row `row` (columns 32q..) or zeros past the last row.
__device__ __forceinline__ void load_quarter(const float* __restrict__ src, int row, int n_rows,
                                             int q, float* x) {
  if (row < n_rows) {
    const float4* p = reinterpret_cast<const float4*>(src + (size_t)row * 128 + 32 * q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = __ldg(p + i);
      x[4 * i] = v.x;
      x[4 * i + 1] = v.y;
      x[4 * i + 2] = v.z;
      x[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = 0.f;
  }
}

// n (8 or 16) values times 2^s as fp16 hi / lo at K columns k0.. of row r of
// a K-major [128 x K] operand image pair.
template <int N>
__device__ __forceinline__ void store_split_scaled(const float* x, float scale, uint8_t* a_hi,
                                                   uint8_t* a_lo, int r, int k0) {
#pragma unroll
  for (int c = 0; c < N / 8; ++c) {
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v0 = x[8 * c + 2 * j] * scale, v1 = x[8 * c + 2 * j + 1] * scale;
      const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const __half l0 = __float2half_rn(__fsub_rn(v0, __half2float(h0)));
      const __half l1 = __float2half_rn(__fsub_rn(v1, __half2float(h1)));
      hv[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lv[j] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    const uint32_t off = sw128_off(r, k0 + 8 * c, kBM);
    *reinterpret_cast<uint4*>(a_hi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(a_lo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

// kind::f16 descriptor: A K-major, B MN-major.
__host__ __device__ constexpr uint32_t idesc_f16_kmn(int m, int n) {
  return (1u << 4) | (1u << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Gradient of the head logits of one row (train/model.py:247-256 through
// autograd): lz = z - logsumexp(z) per head over the legal entries,
// logp = lz_m[a_m] + lz_b[a_b], entropy = -sum(max(lz, lowest) exp(lz)).
//   dL/dlz_k = gl [k == a] - ge exp(lz_k) ([lz_k >= lowest] + max(lz_k, lowest))
//   dL/dz_j  = legal_j * (dL/dlz_j - softmax_j * sum_k dL/dlz_k)
// and dL/dvalue = gv.
__device__ __forceinline__ void head_grad(const float* z, bool live, const uint8_t* mrow,
                                          const uint8_t* brow, int am, int ab, float gl, float ge,
                                          float gv, float* dz) {
  const float lowest = -3.402823466e38f;
#pragma unroll
  for (int o = 0; o < 8; ++o) dz[o] = 0.f;
  if (!live) return;
  float zm[5], mx = lowest;
  bool lg[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    lg[k] = mrow[k] != 0;
    zm[k] = lg[k] ? z[k] : lowest;
    mx = fmaxf(mx, zm[k]);
  }
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 5; ++k) tot += expf(zm[k] - mx);
  const float lse = logf(tot) + mx;
  float G[5], p[5], sg = 0.f;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const float lz = zm[k] - lse;
    p[k] = expf(lz);
    const float cl = fmaxf(lz, lowest);
    G[k] = (k == am ? gl : 0.f) - ge * (p[k] * ((lz >= lowest ? 1.f : 0.f) + cl));
    sg += G[k];
  }
#pragma unroll
  for (int k = 0; k < 5; ++k) dz[k] = lg[k] ? G[k] - p[k] * sg : 0.f;
  const bool b0 = brow[0] != 0, b1 = brow[1] != 0;
  const float zb0 = b0 ? z[5] : lowest, zb1 = b1 ? z[6] : lowest;
  const float mb = fmaxf(zb0, zb1);
  const float lseb = logf(expf(zb0 - mb) + expf(zb1 - mb)) + mb;
  const float l0 = zb0 - lseb, l1 = zb1 - lseb;
  const float p0 = expf(l0), p1 = expf(l1);
  const float G0 = (ab == 0 ? gl : 0.f) - ge * (p0 * ((l0 >= lowest ? 1.f : 0.f) + fmaxf(l0, lowest)));
  const float G1 = (ab == 1 ? gl : 0.f) - ge * (p1 * ((l1 >= lowest ? 1.f : 0.f) + fmaxf(l1, lowest)));
  const float sb = G0 + G1;
  dz[5] = b0 ? G0 - p0 * sb : 0.f;
  dz[6] = b1 ? G1 - p1 * sb : 0.f;
  dz[7] = gv;
}

// A read-only load the compiler keeps in place: the per-layer parameters
// are read again where they are used instead of being held in registers
// across the whole tile loop.
__device__ __forceinline__ float ldg_keep(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// 16 consecutive floats (16-byte aligned) as four 16-byte loads.
__device__ __forceinline__ void ldg16_keep(const float* p, float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[4 * j]), "=f"(v[4 * j + 1]), "=f"(v[4 * j + 2]), "=f"(v[4 * j + 3])
                 : "l"(p + 4 * j));
}

// LayerNorm + affine + ReLU backward for the thread's 32 columns: x holds
// the pre-LN values (-> x-hat), dr the gradient of the ReLU output times
// 2^s (-> dL/dx-hat); the gamma and beta sums of the warp's rows go into
// acc_g, acc_b (reduce-scatter), s1 / s2 are the thread's parts of
// sum(dx-hat) and sum(dx-hat * x-hat).
__device__ __forceinline__ void ln_relu_backward(float* x, float* dr, float mean, float rstd,
                                                 float undo, const float* __restrict__ g,
                                                 const float* __restrict__ b, float& acc_g,
                                                 float& acc_b, float& s1, float& s2) {
  float v[32];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    ldg16_keep(g + 16 * c, v);
    ldg16_keep(b + 16 * c, v + 16);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float xh = (x[16 * c + i] - mean) * rstd;
      const float av = fmaf(xh, v[i], v[16 + i]);
      x[16 * c + i] = xh;
      dr[16 * c + i] = av > 0.f ? dr[16 * c + i] * undo : 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = dr[i];
  acc_b += reduce_scatter32(v);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = dr[i] * x[i];
  acc_g += reduce_scatter32(v);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    ldg16_keep(g + 16 * c, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float dxh = dr[16 * c + i] * v[i];
      dr[16 * c + i] = dxh;
      s1 += dxh;
      s2 = fmaf(dxh, x[16 * c + i], s2);
    }
  }
}

struct TailArgs {
  const float* h;          // saved pre-LN activations [n][128]: h2 (heads) / h1 (trunk)
  const float* dh_in;      // trunk: dL/dh2 [n][128]
  const uint8_t* mm;       // heads: legal moves [n][mm_stride], bomb [n][bm_stride]
  const uint8_t* bm;
  const int64_t* act;      // heads: recorded actions [n][act_stride]
  const float* g;          // heads: [3][n] dL/dlogp, dL/dentropy, dL/dvalue
  const uint32_t* amax;    // heads: max |g|; trunk: max |dL/dh2|
  float* dh_out;           // dL/dh2 (heads) / dL/dh1 (trunk) [n][128]
  float* wpart;            // [grid][out rows][128] per-CTA weight-gradient sums
  float* apart;            // [grid][16 warps][32 lanes][acc] per-thread small sums
  int mm_stride, bm_stride, act_stride;
};

// Both backward kernels run 16 warps, all of them epilogue warps (row r =
// 32 * (warp % 4) + lane, column quarter warp / 4); thread 0 also brings in
// the resident weight image and issues the tile's MMA groups, each after the
// barrier on which all 512 threads announced the operand it reads.  With no
// separate producer and MMA warps every thread may hold 128 registers.
constexpr int kTbThreads = kEpiThreads;

// Wait (bounded) for the last commit thread 0 made, so that no MMA is in
// flight when the TMEM is freed; then free it.
__device__ __forceinline__ void tail_teardown(uint32_t tmem, uint64_t* last, uint32_t parity,
                                              bool pending) {
  if (threadIdx.x == 0 && pending) mbar_wait(last, parity);
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp_id() == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

__global__ void __launch_bounds__(kTbThreads, 1)
k_tail_heads_bwd(TailArgs a, const float* __restrict__ f, const uint8_t* __restrict__ img,
                 int n_rows) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* wbar = (uint64_t*)(smem + kThBytes);
  uint64_t* abar = wbar + 1;     // r2 operand written (512 arrivals)
  uint64_t* ubar = abar + 1;     // u complete
  uint64_t* d1bar = ubar + 1;    // du of heads 0, 1 written (512)
  uint64_t* m2bar = d1bar + 1;   // MMAs on heads 0, 1 complete
  uint64_t* d2bar = m2bar + 1;   // du of head 2 written (512)
  uint64_t* m3bar = d2bar + 1;   // MMAs on head 2 complete
  uint32_t* tmem_slot = (uint32_t*)(m3bar + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* du_exp = (int*)(tmem_slot + 2);
  const int warp = warp_id(), lane = lane_id();
  const int n_tiles = (n_rows + kBM - 1) / kBM;
  uint8_t* wh_hi = smem + kThWh;
  uint8_t* wh_lo = wh_hi + kImgH0Bytes;
  uint8_t* r_hi = smem + kThR;
  uint8_t* r_lo = r_hi + kActB;
  uint8_t* d_hi = smem + kThD;
  uint8_t* d_lo = d_hi + kActB;
  const bool issuer = threadIdx.x == 0;

  if (issuer) {
    mbar_init(wbar, 1);
    mbar_init(abar, kTbThreads);
    mbar_init(ubar, 1);
    mbar_init(d1bar, kTbThreads);
    mbar_init(m2bar, 1);
    mbar_init(d2bar, kTbThreads);
    mbar_init(m3bar, 1);
    *abort_flag = 0;
    // |dL/du| <= 8 max|g| max_u sum_o |Wk2[o][u]| (the logit gradients are at
    // most 2|dL/dlogp| + 4|dL/dentropy|, the value's |dL/dvalue|)
    float colmax = 0.f;
    for (int u = 0; u < 64; ++u) {
      float s0 = 0.f, s1 = 0.f;
      for (int o = 0; o < 5; ++o) s0 += fabsf(f[F_HW2 + o * 64 + u]);
      for (int o = 5; o < 7; ++o) s1 += fabsf(f[F_HW2 + o * 64 + u]);
      colmax = fmaxf(colmax, fmaxf(fmaxf(s0, s1), fabsf(f[F_HW2 + 7 * 64 + u])));
    }
    const float bound = 8.f * __uint_as_float(*a.amax) * colmax;
    const uint32_t bb = __float_as_uint(bound);
    *du_exp = dh_scale_exp(&bb);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(wbar, 2 * kImgH0Bytes);
    for (uint32_t o = 0; o < 2 * kImgH0Bytes; o += 16384)
      bulk_load(wh_hi + o, img + kImgH0 + o, 16384, wbar);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  const uint32_t c_u = 192;                    // u (N = 192), then dr2 (N = 128)
  const uint32_t id_u = idesc_f16(kBM, 192);
  const uint32_t id_dr = idesc_f16_kmn(kBM, 128);
  const uint32_t id_w2 = idesc_f16_mn(kBM, 128), id_w1 = idesc_f16_mn(kBM, 64);
  int committed = 0;                           // thread 0: commits made (3 per tile)
  bool wload = issuer ? mbar_wait(wbar, 0) : true;

  const int qd = warp & 3;
  const int q = warp >> 2;
  const int r = qd * 32 + lane;
  const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
  const uint32_t scr = lane_base + kTbScr;
  const float dscale = pow2f(*du_exp), undo = pow2f(-*du_exp);
  // the thread's small-gradient sums live in TMEM columns of its row's lane
  // (columns kTbAcc + 9q ..), not in registers
  const uint32_t acol = lane_base + kTbAcc + (uint32_t)(kThAcc * q);
  {
    const float z8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    tmem_st8(acol, z8);
    tmem_st1(acol + 8, 0.f);
  }
  bool ok = epi_and(wload);
  for (int tile = blockIdx.x, lt = 0; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
    const uint32_t par = (uint32_t)(lt & 1);
    const int row = tile * kBM + r;
    // E1: LN2 of h2 -> r2 operand
    float x[32], mean, rstd;
    load_quarter(a.h, row, n_rows, q, x);
    ln_stats_quarter(x, q, scr, mean, rstd);
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 gg = __ldg(reinterpret_cast<const float4*>(f + F_LN2G + 32 * q + i));
      const float4 be = __ldg(reinterpret_cast<const float4*>(f + F_LN2B + 32 * q + i));
      x[i] = fmaxf(fmaf((x[i] - mean) * rstd, gg.x, be.x), 0.f);
      x[i + 1] = fmaxf(fmaf((x[i + 1] - mean) * rstd, gg.y, be.y), 0.f);
      x[i + 2] = fmaxf(fmaf((x[i + 2] - mean) * rstd, gg.z, be.z), 0.f);
      x[i + 3] = fmaxf(fmaf((x[i + 3] - mean) * rstd, gg.w, be.w), 0.f);
    }
    store_split_quarter(x, r_hi, r_lo, r, q);
    fence_proxy_async();
    asm volatile("tcgen05.fence::before_thread_sync;");
    mbar_arrive(abar);
    if (issuer) {
      if (mbar_wait(abar, par) && !*abort_flag) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        umma_split_k128(tmem + c_u, r_hi, r_lo, wh_hi, wh_lo, 192, id_u);
        umma_commit(ubar);
        ++committed;
      } else {
        *abort_flag = 1;
      }
    }
    // E2: head outputs and their gradients
    ok = epi_and(mbar_wait(ubar, par) && *abort_flag == 0);
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;");
    float z[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) z[o] = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int u0 = 64 * k + 16 * q;          // this thread's 16 units of head k
      float h[16], w[16];
      tmem_ld16(lane_base + c_u + u0, h);
      ldg16_keep(f + F_HB0 + u0, w);
#pragma unroll
      for (int i = 0; i < 16; ++i) h[i] = fmaxf(__fadd_rn(h[i], w[i]), 0.f);
      const int o_lo = k == 0 ? 0 : (k == 1 ? 5 : 7), o_hi = k == 0 ? 5 : (k == 1 ? 7 : 8);
#pragma unroll
      for (int o = 0; o < 8; ++o) {
        if (o < o_lo || o >= o_hi) continue;
        ldg16_keep(f + F_HW2 + o * 64 + 16 * q, w);
#pragma unroll
        for (int i = 0; i < 16; ++i) z[o] = fmaf(w[i], h[i], z[o]);
      }
    }
    tmem_st8(scr + 16 + 8 * q, z);
    asm volatile("tcgen05.fence::before_thread_sync;");
    epi_sync();
    asm volatile("tcgen05.fence::after_thread_sync;");
    float dz[8];
    {
      float zz[32];
      tmem_ld32(scr + 16, zz);
#pragma unroll
      for (int o = 0; o < 8; ++o)
        z[o] = ((zz[o] + zz[8 + o]) + (zz[16 + o] + zz[24 + o])) + __ldg(f + F_HB2 + o);
      const bool live = row < n_rows;
      const size_t rw = live ? (size_t)row : 0;
      const int64_t am = live ? a.act[rw * a.act_stride] : 0;
      const int64_t ab = live ? a.act[rw * a.act_stride + 1] : 0;
      head_grad(z, live, a.mm + rw * a.mm_stride, a.bm + rw * a.bm_stride,
                (am >= 0 && am < 5) ? (int)am : -1, (ab >= 0 && ab < 2) ? (int)ab : -1,
                live ? a.g[rw] : 0.f, live ? a.g[(size_t)n_rows + rw] : 0.f,
                live ? a.g[2 * (size_t)n_rows + rw] : 0.f, dz);
    }
    // heads 0 and 1: dL/du, the output-layer and hidden-bias sums, du operand.
    // 32-vectors (lane l keeps element l): acc0 = [q0 dz0 | q0 dz1],
    // acc1 = [q0 dz2 | q0 dz3], acc2 = [q0 dz4 | du0], acc3 = [q1 dz5 | q1 dz6],
    // acc4 = [du1 | dz0..7 (quarter 0) | 0], acc5 = [q2 dz7 | du2]
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int u0 = 64 * k + 16 * q;
      float h[16], du[16], v[32];
      tmem_ld16(lane_base + c_u + u0, h);
      ldg16_keep(f + F_HB0 + u0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        h[i] = __fadd_rn(h[i], v[i]);          // pre-ReLU g
        du[i] = 0.f;
      }
#pragma unroll
      for (int o = (k == 0 ? 0 : 5); o < (k == 0 ? 5 : 7); ++o) {
        ldg16_keep(f + F_HW2 + o * 64 + 16 * q, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) du[i] = fmaf(dz[o], v[i], du[i]);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        du[i] = h[i] > 0.f ? du[i] : 0.f;
        h[i] = fmaxf(h[i], 0.f);
      }
      if (k == 0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) { v[i] = h[i] * dz[0]; v[16 + i] = h[i] * dz[1]; }
        tmem_acc(acol + 0, reduce_scatter32(v));
#pragma unroll
        for (int i = 0; i < 16; ++i) { v[i] = h[i] * dz[2]; v[16 + i] = h[i] * dz[3]; }
        tmem_acc(acol + 1, reduce_scatter32(v));
#pragma unroll
        for (int i = 0; i < 16; ++i) { v[i] = h[i] * dz[4]; v[16 + i] = du[i]; }
        tmem_acc(acol + 2, reduce_scatter32(v));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) { v[i] = h[i] * dz[5]; v[16 + i] = h[i] * dz[6]; }
        tmem_acc(acol + 3, reduce_scatter32(v));
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = du[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) { v[16 + i] = q == 0 ? dz[i] : 0.f; v[24 + i] = 0.f; }
        tmem_acc(acol + 4, reduce_scatter32(v));
      }
      store_split_scaled<16>(du, dscale, d_hi, d_lo, r, 64 * k + 16 * q);
    }
    fence_proxy_async();
    asm volatile("tcgen05.fence::before_thread_sync;");
    mbar_arrive(d1bar);
    if (issuer) {
      if (mbar_wait(d1bar, par) && !*abort_flag) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        // dr2 = du(heads 0, 1) Wh0[rows 0..127]: A K-major (K = hidden units),
        // B = Wh0's image read MN-major (N = 128 inputs, K = its rows)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t ao = (uint32_t)(kb * 16384 + kk * 32);
            const uint32_t bo = (uint32_t)((64 * kb + 16 * kk) * 128);
            const uint64_t ah = sw128_desc(d_hi + ao), al = sw128_desc(d_lo + ao);
            const uint64_t bh = sw128_mn_desc(wh_hi + bo, 192 * 128);
            const uint64_t bl = sw128_mn_desc(wh_lo + bo, 192 * 128);
            umma_f16(tmem + c_u, ah, bh, id_dr, (kb | kk) ? 1u : 0u);
            umma_f16(tmem + c_u, ah, bl, id_dr, 1u);
            umma_f16(tmem + c_u, al, bh, id_dr, 1u);
          }
        // dWh0^T[:, 0..127] += r2^T du(heads 0, 1): both operands MN-major
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t o = (uint32_t)(kk * 2048);
          const uint64_t ah = sw128_mn_desc(r_hi + o, 16384), al = sw128_mn_desc(r_lo + o, 16384);
          const uint64_t bh = sw128_mn_desc(d_hi + o, 16384), bl = sw128_mn_desc(d_lo + o, 16384);
          umma_f16(tmem, ah, bh, id_w2, (lt > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tmem, ah, bl, id_w2, 1u);
          umma_f16(tmem, al, bh, id_w2, 1u);
        }
        umma_commit(m2bar);
        ++committed;
      } else {
        *abort_flag = 1;
      }
    }
    // head 2 once the MMAs have released the du operand
    ok = epi_and(mbar_wait(m2bar, par) && *abort_flag == 0);
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;");
    {
      const int u0 = 128 + 16 * q;
      float h[16], du[16], v[32];
      tmem_ld16(lane_base + c_u + u0, h);
      ldg16_keep(f + F_HB0 + u0, v);
      ldg16_keep(f + F_HW2 + 7 * 64 + 16 * q, v + 16);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float g = __fadd_rn(h[i], v[i]);
        h[i] = fmaxf(g, 0.f);
        du[i] = g > 0.f ? dz[7] * v[16 + i] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) { v[i] = h[i] * dz[7]; v[16 + i] = du[i]; }
      tmem_acc(acol + 5, reduce_scatter32(v));
      store_split_scaled<16>(du, dscale, d_hi, d_lo, r, 16 * q);
    }
    fence_proxy_async();
    asm volatile("tcgen05.fence::before_thread_sync;");
    mbar_arrive(d2bar);
    if (issuer) {
      if (mbar_wait(d2bar, par) && !*abort_flag) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        // head 2 (its du in the first K block)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t ao = (uint32_t)(kk * 32);
          const uint32_t bo = (uint32_t)((128 + 16 * kk) * 128);
          const uint64_t ah = sw128_desc(d_hi + ao), al = sw128_desc(d_lo + ao);
          const uint64_t bh = sw128_mn_desc(wh_hi + bo, 192 * 128);
          const uint64_t bl = sw128_mn_desc(wh_lo + bo, 192 * 128);
          umma_f16(tmem + c_u, ah, bh, id_dr, 1u);
          umma_f16(tmem + c_u, ah, bl, id_dr, 1u);
          umma_f16(tmem + c_u, al, bh, id_dr, 1u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t o = (uint32_t)(kk * 2048);
          const uint64_t ah = sw128_mn_desc(r_hi + o, 16384), al = sw128_mn_desc(r_lo + o, 16384);
          const uint64_t bh = sw128_mn_desc(d_hi + o, 16384), bl = sw128_mn_desc(d_lo + o, 16384);
          umma_f16(tmem + 128, ah, bh, id_w1, (lt > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tmem + 128, ah, bl, id_w1, 1u);
          umma_f16(tmem + 128, al, bh, id_w1, 1u);
        }
        umma_commit(m3bar);
        ++committed;
      } else {
        *abort_flag = 1;
      }
    }
    // E3: LN2 backward
    ok = epi_and(mbar_wait(m3bar, par) && *abort_flag == 0);
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;");
    float dr[32];
    tmem_ld32(lane_base + c_u + 32 * q, dr);
    load_quarter(a.h, row, n_rows, q, x);
    float s1 = 0.f, s2 = 0.f, ag = 0.f, ab = 0.f;
    ln_relu_backward(x, dr, mean, rstd, undo, f + F_LN2G + 32 * q, f + F_LN2B + 32 * q, ag, ab,
                     s1, s2);
    tmem_acc(acol + 6, ag);
    tmem_acc(acol + 7, ab);
    tmem_st2(scr + 8 + 2 * q, s1, s2);
    asm volatile("tcgen05.fence::before_thread_sync;");
    epi_sync();
    asm volatile("tcgen05.fence::after_thread_sync;");
    float ss[8];
    tmem_ld8(scr + 8, ss);
    const float m1 = ((ss[0] + ss[2]) + (ss[4] + ss[6])) * (1.f / 128.f);
    const float m2 = ((ss[1] + ss[3]) + (ss[5] + ss[7])) * (1.f / 128.f);
#pragma unroll
    for (int i = 0; i < 32; ++i) dr[i] = (dr[i] - m1 - x[i] * m2) * rstd;
    if (row < n_rows) {
      float4* out = reinterpret_cast<float4*>(a.dh_out + (size_t)row * 128 + 32 * q);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        out[i] = make_float4(dr[4 * i], dr[4 * i + 1], dr[4 * i + 2], dr[4 * i + 3]);
    }
    tmem_acc(acol + 8, reduce_scatter32(dr));
  }
  if (!ok) *abort_flag = 1;
  // per-thread sums, then the dWh0^T accumulator (lane = input, column = unit)
  float* ap = a.apart + (((size_t)blockIdx.x * kEpiWarps + warp) * 32 + lane) * kThAcc;
  {
    float accv[kThAcc];
    tmem_ld8(acol, accv);
    float a8[4];
    tmem_ld4(acol + 8, a8);
    accv[8] = a8[0];
#pragma unroll
    for (int i = 0; i < kThAcc; ++i) ap[i] = accv[i];
  }
  if (ok && blockIdx.x < n_tiles) {
#pragma unroll 1
    for (int c = 0; c < 3; ++c) {
      float v[16];
      tmem_ld16(lane_base + 48 * q + 16 * c, v);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        a.wpart[((size_t)blockIdx.x * 192 + 48 * q + 16 * c + i) * 128 + r] = v[i] * undo;
    }
  }
  uint64_t* lastb = (committed % 3 == 1) ? ubar : (committed % 3 == 2 ? m2bar : m3bar);
  tail_teardown(tmem, lastb, (uint32_t)(((committed - 1) / 3) & 1), !ok && committed > 0);
}

__global__ void __launch_bounds__(kTbThreads, 1)
k_tail_trunk_bwd(TailArgs a, const float* __restrict__ f, const uint8_t* __restrict__ img,
                 int n_rows) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* wbar = (uint64_t*)(smem + kTtBytes);
  uint64_t* abar = wbar + 1;     // r1 and dh2 operands written (512 arrivals)
  uint64_t* m1bar = abar + 1;    // the tile's MMAs complete
  uint32_t* tmem_slot = (uint32_t*)(m1bar + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  const int n_tiles = (n_rows + kBM - 1) / kBM;
  uint8_t* w_hi = smem + kTtW;
  uint8_t* w_lo = w_hi + kImgW1Bytes;
  uint8_t* r_hi = smem + kTtR;
  uint8_t* r_lo = r_hi + kActB;
  uint8_t* d_hi = smem + kTtD;
  uint8_t* d_lo = d_hi + kActB;
  const bool issuer = threadIdx.x == 0;

  if (issuer) {
    mbar_init(wbar, 1);
    mbar_init(abar, kTbThreads);
    mbar_init(m1bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(wbar, 2 * kImgW1Bytes);
    for (uint32_t o = 0; o < 2 * kImgW1Bytes; o += 16384)
      bulk_load(w_hi + o, img + kImgW1 + o, 16384, wbar);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  const uint32_t c_dr = 128;
  const uint32_t id_dr = idesc_f16_kmn(kBM, 128), id_w = idesc_f16_mn(kBM, 128);
  int committed = 0;
  bool wload = issuer ? mbar_wait(wbar, 0) : true;

  const int qd = warp & 3;
  const int q = warp >> 2;
  const int r = qd * 32 + lane;
  const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
  const uint32_t scr = lane_base + 256;        // columns 256..: free in this kernel
  const int dexp = dh_scale_exp(a.amax);
  const float dscale = pow2f(dexp), undo = pow2f(-dexp);
  float acc[kTtAcc] = {0.f, 0.f, 0.f};
  bool ok = epi_and(wload);
  for (int tile = blockIdx.x, lt = 0; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
    const int row = tile * kBM + r;
    float x[32], mean, rstd;
    load_quarter(a.h, row, n_rows, q, x);
    ln_stats_quarter(x, q, scr, mean, rstd);
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 gg = __ldg(reinterpret_cast<const float4*>(f + F_LN1G + 32 * q + i));
      const float4 be = __ldg(reinterpret_cast<const float4*>(f + F_LN1B + 32 * q + i));
      x[i] = fmaxf(fmaf((x[i] - mean) * rstd, gg.x, be.x), 0.f);
      x[i + 1] = fmaxf(fmaf((x[i + 1] - mean) * rstd, gg.y, be.y), 0.f);
      x[i + 2] = fmaxf(fmaf((x[i + 2] - mean) * rstd, gg.z, be.z), 0.f);
      x[i + 3] = fmaxf(fmaf((x[i + 3] - mean) * rstd, gg.w, be.w), 0.f);
    }
    store_split_quarter(x, r_hi, r_lo, r, q);
    load_quarter(a.dh_in, row, n_rows, q, x);
    store_split_scaled<32>(x, dscale, d_hi, d_lo, r, 32 * q);
    fence_proxy_async();
    asm volatile("tcgen05.fence::before_thread_sync;");
    mbar_arrive(abar);
    if (issuer) {
      if (mbar_wait(abar, (uint32_t)(lt & 1)) && !*abort_flag) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        // dr1 = dh2 W1: A K-major (K = outputs), B = W1's image read MN-major
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ao = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
          const uint32_t bo = (uint32_t)(kk * 2048);
          const uint64_t ah = sw128_desc(d_hi + ao), al = sw128_desc(d_lo + ao);
          const uint64_t bh = sw128_mn_desc(w_hi + bo, 16384), bl = sw128_mn_desc(w_lo + bo, 16384);
          umma_f16(tmem + c_dr, ah, bh, id_dr, kk ? 1u : 0u);
          umma_f16(tmem + c_dr, ah, bl, id_dr, 1u);
          umma_f16(tmem + c_dr, al, bh, id_dr, 1u);
        }
        // dW1^T += r1^T dh2: both MN-major, K = the tile's rows
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t o = (uint32_t)(kk * 2048);
          const uint64_t ah = sw128_mn_desc(r_hi + o, 16384), al = sw128_mn_desc(r_lo + o, 16384);
          const uint64_t bh = sw128_mn_desc(d_hi + o, 16384), bl = sw128_mn_desc(d_lo + o, 16384);
          umma_f16(tmem, ah, bh, id_w, (lt > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tmem, ah, bl, id_w, 1u);
          umma_f16(tmem, al, bh, id_w, 1u);
        }
        umma_commit(m1bar);
        ++committed;
      } else {
        *abort_flag = 1;
      }
    }
    ok = epi_and(mbar_wait(m1bar, (uint32_t)(lt & 1)) && *abort_flag == 0);
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;");
    float dr[32];
    tmem_ld32(lane_base + c_dr + 32 * q, dr);
    load_quarter(a.h, row, n_rows, q, x);
    float s1 = 0.f, s2 = 0.f;
    ln_relu_backward(x, dr, mean, rstd, undo, f + F_LN1G + 32 * q, f + F_LN1B + 32 * q, acc[0],
                     acc[1], s1, s2);
    tmem_st2(scr + 8 + 2 * q, s1, s2);
    asm volatile("tcgen05.fence::before_thread_sync;");
    epi_sync();
    asm volatile("tcgen05.fence::after_thread_sync;");
    float ss[8];
    tmem_ld8(scr + 8, ss);
    const float m1 = ((ss[0] + ss[2]) + (ss[4] + ss[6])) * (1.f / 128.f);
    const float m2 = ((ss[1] + ss[3]) + (ss[5] + ss[7])) * (1.f / 128.f);
#pragma unroll
    for (int i = 0; i < 32; ++i) dr[i] = (dr[i] - m1 - x[i] * m2) * rstd;
    if (row < n_rows) {
      float4* out = reinterpret_cast<float4*>(a.dh_out + (size_t)row * 128 + 32 * q);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        out[i] = make_float4(dr[4 * i], dr[4 * i + 1], dr[4 * i + 2], dr[4 * i + 3]);
    }
    acc[2] += reduce_scatter32(dr);
  }
  if (!ok) *abort_flag = 1;
  float* ap = a.apart + (((size_t)blockIdx.x * kEpiWarps + warp) * 32 + lane) * kTtAcc;
#pragma unroll
  for (int i = 0; i < kTtAcc; ++i) ap[i] = acc[i];
  if (ok && blockIdx.x < n_tiles) {
    float v[32];
    tmem_ld32(lane_base + 32 * q, v);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      a.wpart[((size_t)blockIdx.x * 128 + 32 * q + i) * 128 + r] = v[i] * undo;
  }
  tail_teardown(tmem, m1bar, (uint32_t)((committed - 1) & 1), !ok && committed > 0);
}

// Parameter gradients from the per-CTA partial sums, in CTA order
// (deterministic).
//   dWh0: wpart_h [grid][192][128] -> the three head hidden weights
//   dW1:  wpart_t [grid][128][128]
//   small sums: thread (warp 4q + m, lane l) of each CTA holds element l of
//   the 32-vectors built for quarter q.
struct TailGrads {
  float* p[20];            // reference state_dict order (qqt_mlp_param_names)
};

// Destination of the small sum kept by lane l of quarter q's warps in
// accumulator `slot` (kind 0: heads kernel, 1: trunk kernel); nullptr for
// padding.  Heads kernel 32-vectors: slot 0 [q0 dz0 | q0 dz1], 1 [q0 dz2 |
// q0 dz3], 2 [q0 dz4 | du0], 3 [q1 dz5 | q1 dz6], 4 [du1 | dz0..7 (quarter
// 0) | 0], 5 [q2 dz7 | du2], 6 LN2 gamma, 7 LN2 beta, 8 shared.3 bias;
// trunk kernel: 0 LN1 gamma, 1 LN1 beta, 2 shared.0 bias.
__device__ __forceinline__ float* tail_small_dest(const TailGrads& gr, int kind, int q, int l,
                                                  int slot) {
  const int ul = 16 * q + (l & 15);                       // unit within its head
  const bool hi = l >= 16;
  if (kind == 1) return gr.p[slot == 0 ? 2 : (slot == 1 ? 3 : 1)] + 32 * q + l;
  switch (slot) {
    case 0: return gr.p[10] + (hi ? 1 : 0) * 64 + ul;     // move_head.2.weight
    case 1: return gr.p[10] + (hi ? 3 : 2) * 64 + ul;
    case 2: return hi ? gr.p[9] + ul : gr.p[10] + 4 * 64 + ul;   // move_head.0.bias / .2.weight
    case 3: return gr.p[14] + (hi ? 1 : 0) * 64 + ul;     // bomb_head.2.weight
    case 4:
      if (!hi) return gr.p[13] + ul;                      // bomb_head.0.bias
      if (q != 0 || l >= 24) return nullptr;
      return l - 16 < 5 ? gr.p[11] + (l - 16) : (l - 16 < 7 ? gr.p[15] + (l - 21) : gr.p[19]);
    case 5: return hi ? gr.p[17] + ul : gr.p[18] + ul;    // critic.0.bias / critic.2.weight
    case 6: return gr.p[6] + 32 * q + l;                  // shared.4.weight (LN2 gamma)
    case 7: return gr.p[7] + 32 * q + l;                  // shared.4.bias
    default: return gr.p[5] + 32 * q + l;                 // shared.3.bias
  }
}

// One warp per small gradient element: lane j sums CTA-warp partials j,
// j + 32, ... (each CTA's four row-quadrant warps of quarter q) in order,
// then a fixed shuffle tree.
__global__ void k_tail_reduce_small(const float* __restrict__ aph, const float* __restrict__ apt,
                                    int grid, TailGrads gr) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = lane_id();
  constexpr int kHeads = 128 * kThAcc, kAll = kHeads + 128 * kTtAcc;
  if (w >= kAll) return;
  const int kind = w < kHeads ? 0 : 1;
  const int idx = kind ? w - kHeads : w;
  const int nacc = kind ? kTtAcc : kThAcc;
  const int slot = idx % nacc, ql = idx / nacc, q = ql >> 5, l = ql & 31;
  float* dst = tail_small_dest(gr, kind, q, l, slot);
  if (!dst) return;
  const float* ap = kind ? apt : aph;
  float s = 0.f;
  for (int j = lane; j < grid * 4; j += 32)
    s += ap[((((size_t)(j >> 2)) * kEpiWarps + 4 * q + (j & 3)) * 32 + l) * nacc + slot];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) *dst = s;
}

__global__ void k_tail_reduce(const float* __restrict__ wph, const float* __restrict__ wpt,
                              int grid, TailGrads gr) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 192 * 128) {
    float s = 0.f;
    for (int c = 0; c < grid; ++c) s += wph[(size_t)c * 192 * 128 + i];
    const int u = i >> 7, k = i & 127;
    gr.p[8 + 4 * (u >> 6)][(u & 63) * 128 + k] = s;      // move/bomb/critic .0.weight
  }
  if (i < 128 * 128) {
    float s = 0.f;
    for (int c = 0; c < grid; ++c) s += wpt[(size_t)c * 128 * 128 + i];
    gr.p[4][i] = s;                                       // shared.3.weight [out][in]
  }
}

struct TrainWork {
  size_t amax_g, amax_d, dh2, wph, aph, wpt, apt, total;
};

static TrainWork train_work_layout(int n_rows) {
  const int grid = max(1, min((n_rows + kBM - 1) / kBM, sm_count()));
  TrainWork w;
  auto up = [](size_t v) { return (v + 1023) / 1024 * 1024; };
  w.amax_g = 0;
  w.amax_d = 256;
  w.dh2 = 1024;
  w.wph = w.dh2 + up((size_t)n_rows * 128 * 4);
  w.aph = w.wph + up((size_t)grid * 192 * 128 * 4);
  w.wpt = w.aph + up((size_t)grid * kEpiThreads * kThAcc * 4);
  w.apt = w.wpt + up((size_t)grid * 128 * 128 * 4);
  w.total = w.apt + up((size_t)grid * kEpiThreads * kTtAcc * 4);
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
  const int row16 = (int)(row_bytes / 16);
  int lanes = 1;
  while (lanes < 32 && lanes < row16) lanes <<= 1;
  const int64_t threads = (n + 32 / lanes - 1) / (32 / lanes) * 32;
  k_gather_rows<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)src, src_stride_bytes / 16, n_src, idx, n, (uint4*)dst, dst_stride_bytes / 16,
      row16, lanes);
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
                            const int64_t* idx, int64_t n_src, const float* dh1,
                            int32_t n_players, int32_t channels, int32_t hw, int32_t pid,
                            float* dw0, void* work, qqt_stream_t stream) {
  if (!x || !dh1 || !dw0 || !work || n_rows <= 0 || k_in <= 0 || x_stride < k_in ||
      k_in != channels * hw)
    return QQT_E_ARG;
  if (n_rows > (int64_t)0x7fffff00 || (idx && (n_src <= 0 || n_src > (int64_t)0x7fffff00)))
    return QQT_E_LIMIT;
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
      !make_map(&mx, x, (uint64_t)k_in, (uint64_t)(idx ? n_src : n_rows), (uint64_t)x_stride * 2,
                idx ? 1u : (uint32_t)kWgBK))
    return QQT_E_ARG;
  cudaFuncSetAttribute(k_l1_wgrad, cudaFuncAttributeMaxDynamicSharedMemorySize, kWgSmem);
  const int slices = wgrad_slices((int)n_rows, kp);
  const dim3 grid((unsigned)((kp + kWgN - 1) / kWgN), (unsigned)slices);
  float* part = (float*)(wk + L.part);
  k_l1_wgrad<<<grid, kWgThreads, kWgSmem, st>>>(mh, ml, mx, (int)n_rows, kp, part, idx,
                                                 (int)n_src);
  const int64_t n_out = (int64_t)128 * k_in;
  k_wgrad_reduce<<<(unsigned)((n_out + 255) / 256), 256, 0, st>>>(part, slices, kp, k_in, hw, cs,
                                                                 amax, dw0);
  return launch_status();
}

// ---- training forward / tail backward of the MLP (one seat, pack from
// qqt_mlp_pack with n_seats = 1 and the seat's pid)

extern "C" int qqt_mlp_train_forward(const void* pack, const void* obs, int32_t n_rows,
                                     int32_t obs_stride, int32_t k_in, const int64_t* idx,
                                     int64_t n_src, const uint8_t* mm,
                                     int32_t mm_stride, const uint8_t* bm, int32_t bm_stride,
                                     const int64_t* act, int32_t act_stride, float* logp,
                                     float* ent, float* value, float* h1, float* h2,
                                     qqt_stream_t stream) {
  if (!pack || !obs || !mm || !bm || !act || !logp || !ent || !value || !h1 || !h2)
    return QQT_E_ARG;
  if (n_rows <= 0 || k_in <= 0 || obs_stride < k_in || mm_stride < 5 || bm_stride < 2 ||
      act_stride < 2)
    return QQT_E_ARG;
  if ((obs_stride % 8) || ((uintptr_t)obs & 15) || ((uintptr_t)pack & 255) ||
      ((uintptr_t)h1 & 15) || ((uintptr_t)h2 & 15))
    return QQT_E_ALIGN;
  if (idx && (n_src <= 0 || n_src > (int64_t)0x7fffff00)) return QQT_E_LIMIT;
  const MlpPack L = mlp_pack_layout(k_in, 1);
  const uint8_t* pk = (const uint8_t*)pack;
  CUtensorMap ma, mb;
  if (!make_map(&ma, obs, (uint64_t)k_in, (uint64_t)(idx ? n_src : n_rows),
                (uint64_t)obs_stride * 2, idx ? 1u : (uint32_t)kBM))
    return QQT_E_ARG;
  if (!make_map(&mb, pk + L.b_off, (uint64_t)L.kp, 256, (uint64_t)L.kp * 2, 128))
    return QQT_E_ARG;
  SeatOut io;
  memset(&io, 0, sizeof(io));
  io.mm[0] = mm;
  io.bm[0] = bm;
  io.act[0] = const_cast<int64_t*>(act);
  TrainOut tr;
  tr.h1 = h1;
  tr.h2 = h2;
  tr.ent = ent;
  tr.idx = idx;
  tr.n_src = (int)n_src;
  return launch_mlp_fused<128, false, true>(ma, ma, mb, n_rows, L.kp / kBK,
                                            (const float*)(pk + L.f_off), pk + L.img_off, io, 0,
                                            mm_stride, bm_stride, nullptr, act_stride, logp,
                                            value, nullptr, (cudaStream_t)stream, tr);
}

extern "C" uint64_t qqt_mlp_train_work_bytes(int32_t n_rows) {
  if (n_rows <= 0) return 0;
  return train_work_layout(n_rows).total;
}

extern "C" int qqt_mlp_train_backward(const void* pack, int32_t n_rows, int32_t k_in,
                                      const float* h1, const float* h2, const uint8_t* mm,
                                      int32_t mm_stride, const uint8_t* bm, int32_t bm_stride,
                                      const int64_t* act, int32_t act_stride, const float* g,
                                      float* const* grads, float* dh1, void* work,
                                      qqt_stream_t stream) {
  if (!pack || !h1 || !h2 || !mm || !bm || !act || !g || !grads || !dh1 || !work)
    return QQT_E_ARG;
  if (n_rows <= 0 || k_in <= 0 || mm_stride < 5 || bm_stride < 2 || act_stride < 2)
    return QQT_E_ARG;
  for (int i = 1; i < 20; ++i)
    if (!grads[i]) return QQT_E_ARG;
  if (((uintptr_t)pack & 255) || ((uintptr_t)h1 & 15) || ((uintptr_t)h2 & 15) ||
      ((uintptr_t)dh1 & 15) || ((uintptr_t)work & 1023))
    return QQT_E_ALIGN;
  const MlpPack L = mlp_pack_layout(k_in, 1);
  const uint8_t* pk = (const uint8_t*)pack;
  const float* fpar = (const float*)(pk + L.f_off);
  const uint8_t* img = pk + L.img_off;
  const TrainWork W = train_work_layout(n_rows);
  uint8_t* wk = (uint8_t*)work;
  cudaStream_t st = (cudaStream_t)stream;
  const int sms = sm_count();
  const int grid = max(1, min((n_rows + kBM - 1) / kBM, sms));
  if (cudaMemsetAsync(wk, 0, 512, st) != cudaSuccess) return QQT_E_LAUNCH;
  const int64_t ng = 3 * (int64_t)n_rows;
  k_absmax_n<<<(unsigned)max((int64_t)1, min((ng + 255) / 256, (int64_t)sms * 4)), 256, 0, st>>>(
      g, ng, (uint32_t*)(wk + W.amax_g));
  TailArgs a;
  memset(&a, 0, sizeof(a));
  a.h = h2;
  a.mm = mm;
  a.bm = bm;
  a.act = act;
  a.g = g;
  a.amax = (const uint32_t*)(wk + W.amax_g);
  a.dh_out = (float*)(wk + W.dh2);
  a.wpart = (float*)(wk + W.wph);
  a.apart = (float*)(wk + W.aph);
  a.mm_stride = mm_stride;
  a.bm_stride = bm_stride;
  a.act_stride = act_stride;
  cudaFuncSetAttribute(k_tail_heads_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, kThSmem);
  k_tail_heads_bwd<<<grid, kTbThreads, kThSmem, st>>>(a, fpar, img, n_rows);
  const int64_t nd = (int64_t)n_rows * 128;
  k_absmax_n<<<(unsigned)max((int64_t)1, min((nd + 255) / 256, (int64_t)sms * 8)), 256, 0, st>>>(
      (const float*)(wk + W.dh2), nd, (uint32_t*)(wk + W.amax_d));
  TailArgs b;
  memset(&b, 0, sizeof(b));
  b.h = h1;
  b.dh_in = (const float*)(wk + W.dh2);
  b.amax = (const uint32_t*)(wk + W.amax_d);
  b.dh_out = dh1;
  b.wpart = (float*)(wk + W.wpt);
  b.apart = (float*)(wk + W.apt);
  cudaFuncSetAttribute(k_tail_trunk_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, kTtSmem);
  k_tail_trunk_bwd<<<grid, kTbThreads, kTtSmem, st>>>(b, fpar, img, n_rows);
  TailGrads gr;
  for (int i = 0; i < 20; ++i) gr.p[i] = grads[i];
  k_tail_reduce<<<(192 * 128 + 255) / 256, 256, 0, st>>>(
      (const float*)(wk + W.wph), (const float*)(wk + W.wpt), grid, gr);
  k_tail_reduce_small<<<(128 * (kThAcc + kTtAcc) * 32 + 255) / 256, 256, 0, st>>>(
      (const float*)(wk + W.aph), (const float*)(wk + W.apt), grid, gr);
  return launch_status();
}
