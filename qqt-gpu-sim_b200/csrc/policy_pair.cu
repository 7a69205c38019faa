// The MLP policy on SM pairs (tcgen05 cta_group::2): the inference instance
// of k_mlp_fused for large two-seat batches (self-play, N = 256), with each
// 256-row tile served by a cluster of two CTAs on two SMs.
//
// A pair issues one M = 256 MMA per product whose A rows come from both
// CTAs (128 each) and whose N columns are split between them, so each CTA
// streams its own observation rows and half of the first-layer weights (32
// of 48 KB per K step for two seats) and has room for four 48 KB pipeline
// stages instead of two.  The tail (LayerNorm, Linear(128,128), the heads'
// hidden layer) runs the same way (M = 256, each CTA holding half of every
// weight image, 80 of 160 KB).  Measured on one B200 for 32,768 envs x two
// seats: 113.7 us per launch against 127.0 us for k_mlp_fused<256>.  One
// seat gains nothing (39.9 against 38.9 us for 2,816 envs): its layer 1 is
// bound by the tensor pipe and the shared-memory operand reads of its SM,
// which the pair does not divide, and not by the operand stream.
//
// Roles (576 threads per CTA, as in k_mlp_fused): warp 0 lane 0 of each CTA
// streams its operands (TMA, completing on the leader CTA's stage barrier)
// and loads its half of the tail images; warp 1 lane 0 of the leader issues
// every MMA of the pair and commits them to both CTAs' barriers; 16
// epilogue warps per CTA read their own 128 rows from their own TMEM.  No
// load uses cluster multicast (only the commits multicast their barrier
// arrival).  Every wait is bounded; on an abort the MMA issuer stops, every
// wait that can no longer complete runs out, and every thread still reaches
// the closing cluster barrier.

namespace qqt {

// Shared memory: the layer-1 pipeline (7 stages of 32 KB for one seat, 4 of
// 48 KB for two); once layer 1 is done the drained region holds the
// activation operand (hi, lo) and this CTA's half of the tail images.
template <int NT>
struct PairCfg {
  static constexpr int kABytes = kBM * kBK * 2;              // 128 rows x 64 K, fp16
  static constexpr int kBHalf = (NT / 2) * kBK * 2;          // this CTA's half, hi or lo
  static constexpr int kStageBytes = kABytes + 2 * kBHalf;   // 32 KB (NT 128), 48 KB (NT 256)
  static constexpr int kStages = NT == 128 ? 7 : 4;
  static constexpr int kPipeBytes = kStages * kStageBytes;
  static constexpr int kActBytes = kBM * 128 * 2;            // activation operand, hi or lo
  // this CTA's half r of the tail images (K = 128, swizzled): shared.3 rows
  // [64 r, 64 r + 64) hi, lo, then head-hidden rows [96 r, 96 r + 96) hi, lo
  static constexpr int kW1Half = 64 * 128 * 2;
  static constexpr int kH0Half = 96 * 128 * 2;
  static constexpr int kImgHalf = 2 * kW1Half + 2 * kH0Half;  // 80 KB
  static constexpr int kImg = 2 * kActBytes;
  static constexpr int kTail = kImg + kImgHalf;
  static constexpr int kRegion = kPipeBytes > kTail ? kPipeBytes : kTail;
  static constexpr int kBars = kRegion;                      // barriers, TMEM slot, flag
  static constexpr int kSmem = kBars + 256 + 1024 /*align*/;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColH = NT;                      // head hidden accumulator (192)
  static constexpr uint32_t kColScr = NT + 192;              // row-exchange scratch (48)
};
static_assert(PairCfg<128>::kSmem <= 232448 && PairCfg<256>::kSmem <= 232448,
              "pair MLP shared memory over the per-CTA limit");
// barriers (full, empty: kStages each; accb, wbar, abar, dbar), TMEM slot and
// abort flag below byte 192 of the barrier block, the K-tile flags above it
static_assert((2 * PairCfg<128>::kStages + 4) * 8 + 8 <= 192 &&
                  (2 * PairCfg<256>::kStages + 4) * 8 + 8 <= 192,
              "pair barrier block");
static_assert(2 * PairCfg<128>::kImgHalf == (int)kImgBytes, "two halves = the tail images");
static_assert(PairCfg<256>::kColScr + 48 <= PairCfg<256>::kTmemCols, "TMEM columns");

__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive on the barrier at this shared-memory offset in both CTAs of the
// pair once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Tile load into this CTA's shared memory whose completion is counted on
// the barrier `bar` (a shared::cluster address in the pair's leader CTA).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar, void* dst,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// D[tmem] (+)= A * W over K = 128 with the three-term fp16 split, each
// product one M = 256 MMA across the pair (A: each CTA's 128 rows; W: each
// CTA's w_rows rows, at the same shared-memory offsets in both CTAs).
__device__ __forceinline__ void umma_pair_split_k128(uint32_t d_tmem, const uint8_t* a_hi,
                                                     const uint8_t* a_lo, const uint8_t* w_hi,
                                                     const uint8_t* w_lo, int w_rows,
                                                     uint32_t idesc) {
  const uint64_t ah = sw128_desc(a_hi), al = sw128_desc(a_lo);
  const uint64_t wh = sw128_desc(w_hi), wl = sw128_desc(w_lo);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t oa = (uint64_t)(((kk >> 2) * kBM * 128 + (kk & 3) * 32) >> 4);
    const uint64_t ow = (uint64_t)(((kk >> 2) * w_rows * 128 + (kk & 3) * 32) >> 4);
    umma_f16_pair(d_tmem, ah + oa, wh + ow, idesc, kk > 0 ? 1u : 0u);
    umma_f16_pair(d_tmem, ah + oa, wl + ow, idesc, 1u);
    umma_f16_pair(d_tmem, al + oa, wh + ow, idesc, 1u);
  }
}

// The two halves of the tail images from the f32 parameters, one thread per
// (row, k): half r holds shared.3 rows [64 r, 64 r + 64) and head-hidden
// rows [96 r, 96 r + 96), fp16 hi / lo, each a swizzled K-major K = 128
// image of its own row count.
__global__ void k_mlp_pack_pair_images(HeadParams hp, uint8_t* __restrict__ img) {
  using G = PairCfg<128>;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 192 * 128) return;
  const int n = i >> 7, k = i & 127;
  if (n < 128) {
    const float v = hp.w1[n * 128 + k];                  // [out][in]: K-major already
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    uint8_t* base = img + (n >> 6) * G::kImgHalf;
    *reinterpret_cast<__half*>(base + sw128_off(n & 63, k, 64)) = hi;
    *reinterpret_cast<__half*>(base + G::kW1Half + sw128_off(n & 63, k, 64)) = lo;
  }
  const float v = n < 64 ? hp.mw0[n * 128 + k]
                         : (n < 128 ? hp.bw0[(n - 64) * 128 + k] : hp.cw0[(n - 128) * 128 + k]);
  const __half hi = __float2half_rn(v);
  const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
  const int half = n / 96, nl = n - half * 96;
  uint8_t* base = img + half * G::kImgHalf + 2 * G::kW1Half;
  *reinterpret_cast<__half*>(base + sw128_off(nl, k, 96)) = hi;
  *reinterpret_cast<__half*>(base + G::kH0Half + sw128_off(nl, k, 96)) = lo;
}

// tm_a: the observation rows (box 128 rows); tm_b: the packed first-layer
// weights, hi rows [0, NT) then lo rows [NT, 2 NT) (box NT / 2 rows);
// img: the two image halves of k_mlp_pack_pair_images.
template <int NT>
__global__ void __launch_bounds__(kMlpThreads, 1)
k_mlp_pair(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
           int n_rows, int k_tiles, const float* __restrict__ f, const uint8_t* __restrict__ img,
           SeatOut io, int mm_stride, int bm_stride, const float* __restrict__ u, int act_stride,
           float* __restrict__ logp_out, float* __restrict__ value_out,
           float* __restrict__ logits_out, uint32_t test_wait, const uint4* __restrict__ tiles) {
  using G = PairCfg<NT>;
  constexpr int S = NT / 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + G::kBars);   // leader: stage landed (both CTAs)
  uint64_t* empty = full + G::kStages;   // stage consumed (commit, both CTAs)
  uint64_t* accb = empty + G::kStages;   // layer 1 complete (commit, both CTAs)
  uint64_t* wbar = accb + 1;             // this CTA's image half landed
  uint64_t* abar = wbar + 1;             // leader: both CTAs' activation operands written
  uint64_t* dbar = abar + 1;             // tail MMA group complete (commit, both CTAs)
  uint32_t* tmem_slot = (uint32_t*)(dbar + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  uint4* kpart = (uint4*)(smem + G::kBars + 192);   // K-tile flags, one word set per warp
  const int warp = warp_id(), lane = lane_id();
  const int rank = (int)cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int m0 = (2 * pair + rank) * kBM;
  // a second CTA wholly past the end (odd tile count) streams the last
  // tile's rows again; its own rows are never written
  const int m_load = min(m0, (n_rows - 1) / kBM * kBM);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    for (int s = 0; s < G::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    mbar_init(wbar, 1);
    mbar_init(abar, 2);
    mbar_init(dbar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    // one warp of each CTA of the pair allocates the pair's TMEM collectively
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(G::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  // both CTAs OR the flags of the pair's 256 rows, so both run the same tiles
  if (warp >= 2 && warp < 6) ktile_flags_part(tiles, 2 * pair * kBM, 2 * pair * kBM + 2 * kBM,
                                              n_rows, kpart);
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  // both CTAs' barriers are initialised before any remote arrival or load
  cluster_arrive();
  cluster_wait();
  const uint32_t tmem = *tmem_slot;
  if (test_wait) {
    // failure-path check (qqt_test_set_wait_polls): a bounded wait of
    // test_wait polls on the image barrier, which nothing completes before
    // the loads are issued, runs out in both CTAs; both then take the abort
    // path before anything is issued
    if (threadIdx.x == 0 && !mbar_wait(wbar, 0, test_wait)) *abort_flag = 1;
    __syncthreads();
  }

  if (warp == 0) {
    const uint64_t kmask = ktile_mask(kpart, k_tiles);
    if (lane == 0) {
      // ---------------- producer (both CTAs)
      int issued = 0;
      bool img_issued = false;
      // pairs start at different K tiles so that at any time they read
      // different lines of the shared weight stream from L2
      const int k0 = (int)(((unsigned)pair * 7u) % (unsigned)k_tiles);
      const int n_run = ktile_count(kmask, 0, k_tiles, k0);
      int kt_src = k0;
      for (int j = 0, kt = 0; j < k_tiles && !*abort_flag;
           ++j, kt_src = kt_src + 1 == k_tiles ? 0 : kt_src + 1) {
        if (j > 0 && !ktile_in(kmask, kt_src)) continue;   // zero in every row of the pair
        const int s = kt % G::kStages;
        if (kt >= G::kStages && !mbar_wait(&empty[s], ((kt / G::kStages) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * G::kStageBytes;
        const uint32_t fb = dsmem_addr(&full[s], 0);
        const int kx = kt_src * kBK;
        // the leader's stage barrier counts both CTAs' bytes
        if (leader) mbar_expect_tx(&full[s], 2 * G::kStageBytes);
        tma_load_2d_pair(&tm_a, fb, st, kx, m_load);
        tma_load_2d_pair(&tm_b, fb, st + G::kABytes, kx, rank * (NT / 2));
        tma_load_2d_pair(&tm_b, fb, st + G::kABytes + G::kBHalf, kx, NT + rank * (NT / 2));
        issued = ++kt;
      }
      // every stage this CTA issued is consumed before the CTA may exit
      // (the leader commits each stage's empty barrier in both CTAs)
      for (int kt = max(0, issued - G::kStages); kt < issued; ++kt)
        if (!mbar_wait(&empty[kt % G::kStages], (kt / G::kStages) & 1)) *abort_flag = 1;
      if (issued == n_run && !*abort_flag) {
        // the stages' last MMAs are done (each commit covers every earlier
        // MMA): the drained region takes the images
        mbar_expect_tx(wbar, G::kImgHalf);
        const uint8_t* src = img + (size_t)rank * G::kImgHalf;
        for (uint32_t o = 0; o < (uint32_t)G::kImgHalf; o += 16384)
          bulk_load(smem + G::kImg + o, src + o, 16384, wbar);
        img_issued = true;
      }
      if (img_issued && !mbar_wait(wbar, 0)) *abort_flag = 1;
    }
  } else if (warp == 1) {
    const uint64_t kmask = ktile_mask(kpart, k_tiles);
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (the leader, for the pair)
      const uint32_t idesc1 = idesc_f16(2 * kBM, NT);
      // the producers' tile sequence: its length is all this loop needs
      const int n_run = ktile_count(kmask, 0, k_tiles, (int)(((unsigned)pair * 7u) % (unsigned)k_tiles));
      bool ok = true;
      for (int kt = 0; kt < n_run; ++kt) {
        const int s = kt % G::kStages;
        if (*abort_flag || !mbar_wait(&full[s], (kt / G::kStages) & 1)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint8_t* st = smem + s * G::kStageBytes;
        const uint64_t da = sw128_desc(st);
        const uint64_t dh = sw128_desc(st + G::kABytes);
        const uint64_t dl = sw128_desc(st + G::kABytes + G::kBHalf);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);   // 32 bytes per K = 16 step
          umma_f16_pair(tmem, da + off, dh + off, idesc1, (kt > 0 || kk > 0) ? 1u : 0u);
          umma_f16_pair(tmem, da + off, dl + off, idesc1, 1u);
        }
        umma_commit_pair(&empty[s]);
      }
      umma_commit_pair(accb);   // fires once every issued MMA has completed
      // tail, per seat: layer 2 (D overwrites the seat's layer-1 columns,
      // already read), then the heads' hidden layer.  Each group waits for
      // both CTAs' activation operands; an epilogue arrives only after its
      // CTA's image half landed, so the images are in place too.
      const uint32_t id2 = idesc_f16(2 * kBM, 128), id3 = idesc_f16(2 * kBM, 192);
      const uint8_t* a_hi = smem;
      const uint8_t* a_lo = smem + G::kActBytes;
      const uint8_t* im = smem + G::kImg;
      int committed = 0;
      for (int s = 0; s < S && ok; ++s) {
        if (*abort_flag || !mbar_wait_cluster(abar, (2 * s) & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;");
        umma_pair_split_k128(tmem + 128 * s, a_hi, a_lo, im, im + G::kW1Half, 64, id2);
        umma_commit_pair(dbar);
        ++committed;
        if (*abort_flag || !mbar_wait_cluster(abar, (2 * s + 1) & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;");
        umma_pair_split_k128(tmem + G::kColH, a_hi, a_lo, im + 2 * G::kW1Half,
                             im + 2 * G::kW1Half + G::kH0Half, 96, id3);
        umma_commit_pair(dbar);
        ++committed;
      }
      if (!ok) {
        *abort_flag = 1;
        // the MMAs already issued complete before the pair may exit
        mbar_wait(accb, 0);
        if (committed > 0) mbar_wait(dbar, (committed - 1) & 1);
      }
    }
  } else {
    // ---------------- epilogue: row r = 32 * (warp % 4) + lane of this CTA,
    // columns 32 * quarter .. + 31 of each 128-wide layer
    const int qd = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int r = qd * 32 + lane;
    const int row = m0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    const uint32_t scr = lane_base + G::kColScr;
    uint8_t* a_hi = smem;
    uint8_t* a_lo = smem + G::kActBytes;
    const uint32_t abar_lead = dsmem_addr(abar, 0);
    const bool elected = warp == 2 && lane == 0;
    // sampling inputs of this row (the thread of quarter 0 samples it)
    SampleIn sin[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
      sin[s] = SampleIn{0u, 0.f, 0.f};
      if (quarter == 0 && row < n_rows)
        sin[s] = sample_load(row, s, n_rows, io.mm[s], mm_stride, io.bm[s], bm_stride, u);
    }
    // the leader always commits accb, also after an abort: waiting for it
    // keeps the CTA resident until that arrival has landed
    bool ok = mbar_wait(accb, 0);
    ok = epi_and(ok && *abort_flag == 0);
    // layer 1 is done: a kernel launched as this one's programmatic
    // dependent (the simulator step) may start staging its state now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;");
    // this CTA's activation operand is written: the generic-proxy stores
    // are made visible to the tensor cores, the TMEM reads of the columns
    // the next MMA overwrites are ordered before it, and one thread of the
    // CTA arrives on the leader's operand barrier -- the first time only
    // once this CTA's image half has landed, so that the leader's wait
    // covers the images too
    auto operand_ready = [&](bool first) -> bool {
      fence_proxy_async();
      asm volatile("tcgen05.fence::before_thread_sync;");
      bool good = true;
      if (first) good = epi_and(mbar_wait(wbar, 0) && *abort_flag == 0);
      else epi_sync();
      if (elected && good) mbar_arrive_remote(abar_lead);
      return good;
    };
#pragma unroll 1
    for (int s = 0; s < S && ok; ++s) {
      float x[32];
      // LN1 over the seat's layer-1 pre-activations
      tmem_ld32(lane_base + 128 * s + 32 * quarter, x);
      bias_ln_relu_quarter(x, quarter, scr, f + F_B0 + 128 * s, f + F_LN1G, f + F_LN1B);
      store_split_quarter(x, a_hi, a_lo, r, quarter);
      ok = operand_ready(s == 0);
      if (!ok) break;
      // LN2 over layer 2
      ok = epi_and(mbar_wait(dbar, (2 * s) & 1) && *abort_flag == 0);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;");
      tmem_ld32(lane_base + 128 * s + 32 * quarter, x);
      bias_ln_relu_quarter(x, quarter, scr + 8, f + F_B1, f + F_LN2G, f + F_LN2B);
      store_split_quarter(x, a_hi, a_lo, r, quarter);
      operand_ready(false);
      // head hidden units -> this quarter's partial output logits
      ok = epi_and(mbar_wait(dbar, (2 * s + 1) & 1) && *abort_flag == 0);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;");
      float z[8];
#pragma unroll
      for (int o = 0; o < 8; ++o) z[o] = 0.f;
      head_out_quarter(lane_base + G::kColH, quarter, f, z);
      // the four quarters' partial logits through the row's TMEM lane
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
          sample_write(z, row, s, n_rows, sin[s], io.act[s], act_stride, logp_out, value_out,
                       logits_out);
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  // neither CTA leaves (nor frees the pair's TMEM) while the pair's MMAs may
  // still read its shared memory or write its TMEM
  asm volatile("tcgen05.fence::before_thread_sync;");
  cluster_arrive();
  cluster_wait();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(G::kTmemCols));
  }
}

// Pair launches serve batches large enough that k_mlp_fused runs without a
// split-K cluster; QQT_MLP_PAIR=0 turns them off.
static bool mlp_pair_enabled() {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("QQT_MLP_PAIR");
    env = (e && e[0] == '0') ? 0 : 1;
  }
  return env == 1;
}

template <int NT>
static int launch_mlp_pair(const CUtensorMap& ma, const CUtensorMap& mb, int n_rows, int k_tiles,
                           const float* f, const uint8_t* img, const SeatOut& io, int mm_stride,
                           int bm_stride, const float* u, int act_stride, float* logp,
                           float* value, float* logits, cudaStream_t st,
                           const uint4* tiles = nullptr) {
  using G = PairCfg<NT>;
  auto kern = k_mlp_pair<NT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  const int m_tiles = (n_rows + kBM - 1) / kBM;
  const int pairs = (m_tiles + 1) / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kMlpThreads, 1, 1);
  cfg.dynamicSmemBytes = G::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const uint32_t test_wait = g_test_wait_polls.load(std::memory_order_relaxed);
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, n_rows, k_tiles, f, img, io, mm_stride, bm_stride, u,
                         act_stride, logp, value, logits, test_wait, tiles) != cudaSuccess)
    return QQT_E_LAUNCH;
  return launch_status();
}

}  // namespace qqt
