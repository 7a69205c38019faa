// Danger map + shared fp16 observation + legal masks, and the rule bots.
//
// k_observe: one block per tile of 8 envs, one warp per env.
//   danger: stage A (chain correction among bombs) and stage B, both as
//   scatters along each bomb's rays; the observation row is written straight
//   to global memory (consecutive lanes, consecutive cells of a channel).
// k_astar: warp per env; the two path fields share one warp (row / column
//   sweeps to a fixed point, exactly the reference's Bellman-Ford limit).

#include <type_traits>

#include "qqt_common.cuh"

namespace qqt {


// One seat's masks and action rows: row e at base + e * stride.
struct SeatIO {
  const uint8_t* mm;
  const uint8_t* bm;
  int64_t* act;
  int mm_stride, bm_stride, act_stride;
};

struct PInfo {
  float y, x, sw[4];
  int sc[4];
  int flat, alive, live;
  float inv, avail, capv;
  int64_t bombs_cap;
};

// Per-warp scratch of k_observe: stage-A weights and bomb list, then one
// observation row staged in shared memory (the stage-A front/spread arrays
// are dead by then and share its space), then the per-player values.
struct ObsLayout {
  size_t cur, bombs, fs, pinfo, dng, total;
};

__host__ __device__ inline size_t a16(size_t x) { return (x + 15) & ~(size_t)15; }

// Per-warp scratch of k_observe: stage-A weights, bomb list, front + spread,
// player info, the danger map.  The observation row itself is written
// straight to global memory.
__host__ __device__ inline ObsLayout obs_layout(int cells) {
  ObsLayout L;
  L.cur = 0;
  L.bombs = a16((size_t)cells * 4);
  L.fs = a16(L.bombs + (size_t)cells * 2);
  L.pinfo = a16(L.fs + (size_t)cells * 8);
  L.dng = a16(L.pinfo + QQT_MAX_P * sizeof(PInfo));
  L.total = a16(L.dng + (size_t)cells * 4);
  return L;
}

template <class T>
__device__ __forceinline__ T to_obs(float v);
template <>
__device__ __forceinline__ float to_obs<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_obs<__half>(float v) { return __float2half_rn(v); }

// Fuse tables (bit-identical to computing the IEEE division / weight per cell).
struct FuseTables {
  float weight[32], norm[32];
  float capv[32];   // i / obs_growth_bombs_max, the observation's bomb-cap value
};

// One env's observation row, masks and (optionally) danger map from its
// staged planes (sim/obs.py:25-229), for the warp that owns the env.  Inputs:
// dng = the env's danger map (sim/blast.py:158-317), live_p = live bombs of
// player p, and for lanes < P that player's position, alive flag,
// invulnerability and bomb cap.  Lane l computes cell l, l+32, ... of every
// channel (consecutive lanes, consecutive elements); the row goes straight to
// global memory, or, given a 16-byte aligned per-warp `stage` of obs_stride
// elements, into shared memory first and out as 16-byte stores.  Staged
// fp16 rows may also report which of their 64-entry K tiles hold a nonzero
// (`tiles`, four words per row: tile t is bit min(t >> 2, 31) of word t & 3,
// the flags the MLP policy uses to skip zero tiles).
template <class T, bool STAGED = false, int NP = 0, int G = 0>
__device__ inline void observe_env(const QqtCfg& cfg, const Env& v, int e, PInfo* pi,
                                   const float* dng, int live_p, float py, float px,
                                   bool alive_p, int64_t inv_p, int64_t bcap_p, int64_t t_e,
                                   const FuseTables& ft, void* obs, float* danger_out,
                                   uint8_t* mm, uint8_t* bm, T* stage = nullptr,
                                   uint32_t* tiles = nullptr) {
  const int h = G > 0 ? G : cfg.height, w = G > 0 ? G : cfg.width, C = h * w;
  const int P = NP > 0 ? NP : cfg.n_players;
  const int lane = lane_id();
  const int nch = cfg.obs_channels;
  if (STAGED) __syncwarp();   // the staging area reuses scratch read just before
  QQT_PH(2, 18, STAGED && (blockIdx.x & 3) == 0 && lane == 0);
  if (lane < P) {
    const int p = lane;
    PInfo q;
    q.y = py;
    q.x = px;
    q.alive = alive_p;
    q.live = live_p;
    const float g = q.alive ? 1.f : 0.f;
    const float fy = fminf(fmaxf(__fsub_rn(q.y, 0.5f), 0.f), (float)(h - 1));
    const float fx = fminf(fmaxf(__fsub_rn(q.x, 0.5f), 0.f), (float)(w - 1));
    const int y0 = min(max((int)floorf(fy), 0), h - 1), x0 = min(max((int)floorf(fx), 0), w - 1);
    const int y1 = min(y0 + 1, h - 1), x1 = min(x0 + 1, w - 1);
    const float wy = fminf(fmaxf(__fsub_rn(fy, (float)y0), 0.f), 1.f);
    const float wx = fminf(fmaxf(__fsub_rn(fx, (float)x0), 0.f), 1.f);
    const float wys[2] = {__fsub_rn(1.f, wy), wy}, wxs[2] = {__fsub_rn(1.f, wx), wx};
    const int ys[2] = {y0, y1}, xs[2] = {x0, x1};
#pragma unroll
    for (int a2 = 0; a2 < 2; ++a2)
#pragma unroll
      for (int b2 = 0; b2 < 2; ++b2) {
        q.sc[a2 * 2 + b2] = ys[a2] * w + xs[b2];
        q.sw[a2 * 2 + b2] = __fmul_rn(__fmul_rn(wys[a2], wxs[b2]), g);
      }
    q.flat = center_cell(q.y, q.x, h, w);
    q.inv = (inv_p > 0 && q.alive) ? 1.f : 0.f;
    q.bombs_cap = bcap_p;
    const float cap = fmaxf((float)q.bombs_cap, 1.f);
    const float avail = fmaxf((float)(q.bombs_cap - (int64_t)q.live), 0.f);
    q.avail = __fmul_rn(__fdiv_rn(avail, cap), g);
    const int64_t ci = q.bombs_cap > 1 ? q.bombs_cap : 1;   // cap as an integer
    q.capv = __fmul_rn(ci < 32 ? ft.capv[ci] : __fdiv_rn(cap, cfg.obs_growth_bombs_max), g);
    pi[p] = q;
  }
  __syncwarp();   // PInfo visible
  QQT_PH(2, 19, STAGED && (blockIdx.x & 3) == 0 && lane == 0);

  const float tv = __fdiv_rn((float)t_e, cfg.max_steps_f);
  T* const grow = obs ? (T*)obs + (size_t)e * cfg.obs_stride : nullptr;
  if (STAGED) {
    // staged row: zero it, write the dense channels cell by cell and the
    // sparse ones (position splats, values at each player's cell) at their
    // cells, then move it out as 16-byte stores (row stride and base are
    // 16-byte aligned: checked by the entry points)
    const int n16 = (int)((size_t)cfg.obs_stride * sizeof(T) / 16);
    uint4* s4 = reinterpret_cast<uint4*>(stage);
#pragma unroll 4
    for (int k = lane; k < n16; k += 32) s4[k] = make_uint4(0, 0, 0, 0);
    __syncwarp();
    QQT_PH(2, 20, STAGED && (blockIdx.x & 3) == 0 && lane == 0);
    const T tvh = to_obs<T>(tv);
    const bool extra = nch > 2 * P + 3;
#pragma unroll
    for (int c = lane; c < C; c += 32) {
      const float d = dng[c];
      if (danger_out) danger_out[(size_t)e * C + c] = d;
      const int f = v.fuse[c], o = v.owner[c];
      if (f > 0 && o >= 0 && o < P)     // own-bomb fuse channel of the owner
        stage[(P + o) * C + c] = to_obs<T>(f < 32 ? ft.norm[f] : __fdiv_rn((float)f, cfg.fuse_f));
      if (v.wall[c] | v.brick[c]) stage[2 * P * C + c] = to_obs<T>(1.f);
      stage[(2 * P + 1) * C + c] = to_obs<T>(d);
      stage[(2 * P + 2) * C + c] = tvh;
      if (extra && v.crate[c]) stage[(2 * P + 3) * C + c] = to_obs<T>(1.f);
    }
    if (lane < P) {
      const PInfo& q = pi[lane];
      // splat cell sc[m]: the sum over the corners that land on it, in corner
      // order from 0 (the reference's four scatter_add calls)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        bool first = true;
#pragma unroll
        for (int m2 = 0; m2 < m; ++m2) first = first && q.sc[m2] != q.sc[m];
        if (!first) continue;
        float sv = 0.f;
#pragma unroll
        for (int m2 = m; m2 < 4; ++m2)
          if (q.sc[m2] == q.sc[m]) sv = __fadd_rn(sv, q.sw[m2]);
        stage[lane * C + q.sc[m]] = to_obs<T>(sv);
      }
      if (extra) {
        stage[(2 * P + 4 + lane) * C + q.flat] = to_obs<T>(q.inv);
        stage[(3 * P + 4 + lane) * C + q.flat] = to_obs<T>(q.avail);
        stage[(4 * P + 4 + lane) * C + q.flat] = to_obs<T>(q.capv);
      }
    }
    __syncwarp();
    QQT_PH(2, 21, STAGED && (blockIdx.x & 3) == 0 && lane == 0);
    uint4* dst = reinterpret_cast<uint4*>(grow);
    if (sizeof(T) == 2 && tiles) {
      // chunk k = lane + 32 i (eight entries) lies in K tile k >> 3 =
      // 4 i + (lane >> 3): lane group g = lane >> 3 sees only the tiles of
      // word g, tile 4 i + g at bit i (bit 31 from i = 31 on)
      uint32_t acc = 0, bit = 1;
#pragma unroll 4
      for (int k = lane; k < n16; k += 32) {
        const uint4 x = s4[k];
        dst[k] = x;
        if ((x.x | x.y) | (x.z | x.w)) acc |= bit;
        bit = bit == 0x80000000u ? bit : bit << 1;
      }
      acc |= __shfl_xor_sync(QQT_FULL, acc, 1);
      acc |= __shfl_xor_sync(QQT_FULL, acc, 2);
      acc |= __shfl_xor_sync(QQT_FULL, acc, 4);
      if ((lane & 7) == 0) tiles[(size_t)e * 4 + (lane >> 3)] = acc;
    } else {
#pragma unroll 4
      for (int k = lane; k < n16; k += 32) dst[k] = s4[k];
      if (tiles && lane < 4) tiles[(size_t)e * 4 + lane] = ~0u;
    }
    QQT_PH(2, 22, STAGED && (blockIdx.x & 3) == 0 && lane == 0);
  } else if (obs || danger_out) {
    T* row = grow;
    for (int c = lane; c < C; c += 32) {
      const float d = dng[c];
      if (danger_out) danger_out[(size_t)e * C + c] = d;
      if (!obs) continue;
      const int f = v.fuse[c], o = v.owner[c];
      const float fn = f > 0 ? (f < 32 ? ft.norm[f] : __fdiv_rn((float)f, cfg.fuse_f)) : 0.f;
      for (int p = 0; p < P; ++p) {
        const PInfo& q = pi[p];
        float sv = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m)
          if (q.sc[m] == c) sv = __fadd_rn(sv, q.sw[m]);
        row[p * C + c] = to_obs<T>(sv);
        row[(P + p) * C + c] = to_obs<T>((o == p && f > 0) ? fn : 0.f);
      }
      row[2 * P * C + c] = to_obs<T>((v.wall[c] | v.brick[c]) ? 1.f : 0.f);
      row[(2 * P + 1) * C + c] = to_obs<T>(d);
      row[(2 * P + 2) * C + c] = to_obs<T>(tv);
      if (nch > 2 * P + 3) {
        row[(2 * P + 3) * C + c] = to_obs<T>(v.crate[c] ? 1.f : 0.f);
        // invulnerability flag, available / cap bombs: at each player's cell
        for (int p = 0; p < P; ++p) {
          const PInfo& q = pi[p];
          const bool at = q.flat == c;
          row[(2 * P + 4 + p) * C + c] = to_obs<T>(at ? q.inv : 0.f);
          row[(3 * P + 4 + p) * C + c] = to_obs<T>(at ? q.avail : 0.f);
          row[(4 * P + 4 + p) * C + c] = to_obs<T>(at ? q.capv : 0.f);
        }
        for (int ch = 5 * P + 4; ch < nch; ++ch) row[ch * C + c] = to_obs<T>(0.f);
      }
    }
    if (obs)
      for (int i = nch * C + lane; i < cfg.obs_stride; i += 32) row[i] = to_obs<T>(0.f);
  }

  if (mm) {
    if (lane < 4 * P) {
      const int p = lane >> 2, d = lane & 3;
      const PInfo& q = pi[p];
      const float dv = (d & 1) ? cfg.step_len : -cfg.step_len;
      // one probe per lane: d < 2 moves along the rows, else along the columns
      const bool vert = d < 2;
      const float cq = vert ? q.y : q.x, oq = vert ? q.x : q.y;
      const float nc = resolve_axis(v, __fadd_rn(cq, dv), dv, oq, q.y, q.x, cfg.radius, vert);
      const bool moved = fabsf(__fsub_rn(nc, cq)) > cfg.move_eps2;
      mm[((size_t)e * P + p) * 5 + d] = q.alive ? (moved ? 1 : 0) : 1;
    } else if (lane < 5 * P) {
      mm[((size_t)e * P + (lane - 4 * P)) * 5 + 4] = 1;
    }
  }
  if (bm && lane < P) {
    const PInfo& q = pi[lane];
    const bool under = v.fuse[q.flat] > 0;
    const bool under_b = under || v.brick[q.flat];
    const bool ok = !under && !under_b && (int64_t)q.live < q.bombs_cap;
    bm[((size_t)e * P + lane) * 2 + 0] = 1;
    bm[((size_t)e * P + lane) * 2 + 1] = q.alive ? (ok ? 1 : 0) : 1;
  }
  __syncwarp();
}

// Live bombs (fuse > 0) of player `lane` for lanes < P (0 elsewhere),
// warp-wide: one ballot per player and 32 cells.
__device__ inline int live_count_of_lane(const Env& v, int P) {
  int live[QQT_MAX_P] = {0, 0, 0, 0};
  for (int base = 0; base < v.cells; base += 32) {
    const int c = base + lane_id();
    const int f = c < v.cells ? v.fuse[c] : 0, o = c < v.cells ? v.owner[c] : -1;
#pragma unroll
    for (int q = 0; q < QQT_MAX_P; ++q)
      if (q < P) live[q] += __popc(__ballot_sync(QQT_FULL, f > 0 && o == q));
  }
  int mine = 0;
#pragma unroll
  for (int q = 0; q < QQT_MAX_P; ++q)
    if (lane_id() == q) mine = live[q];
  return mine;
}

__device__ inline void fuse_tables(FuseTables& ft, float fuse_f, float growth_bombs_max) {
  if (threadIdx.x < 32) {
    ft.weight[threadIdx.x] = fuse_weight(threadIdx.x, fuse_f);
    ft.norm[threadIdx.x] = __fdiv_rn((float)threadIdx.x, fuse_f);
    ft.capv[threadIdx.x] = __fdiv_rn((float)threadIdx.x, growth_bombs_max);
  }
}

template <bool F32OUT>
__global__ void __launch_bounds__(QQT_NWARP * 32, 4)
k_observe(QqtCfg cfg, QqtState st, void* obs, float* danger_out, uint8_t* mm, uint8_t* bm) {
  using T = typename std::conditional<F32OUT, float, __half>::type;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ FuseTables ft;
  const int h = cfg.height, w = cfg.width, C = h * w, N = cfg.n_envs, P = cfg.n_players;
  const int e0 = blockIdx.x * QQT_TILE_E;
  fuse_tables(ft, cfg.fuse_f, cfg.obs_growth_bombs_max);
  Tile tile = carve_tile(smem, C);
  load_tile(tile, st, N, e0, PL_WALL | PL_BRICK | PL_CRATE | PL_OWNER | PL_FUSE | PL_BLAST);
  __syncthreads();
  const ObsLayout L = obs_layout(C);
  uint8_t* wb = smem + tile_bytes(C) + (size_t)warp_id() * L.total;
  DangerScratch ds;
  ds.cur = (float*)(wb + L.cur);
  ds.bombs = (uint16_t*)(wb + L.bombs);
  ds.front = (float*)(wb + L.fs);
  ds.spread = ds.front + C;
  PInfo* pi = (PInfo*)(wb + L.pinfo);
  float* dng = (float*)(wb + L.dng);
  const int lane = lane_id();

  for (int s = warp_id(); s < QQT_TILE_E; s += QQT_NWARP) {
    const int e = e0 + s;
    if (e >= N) break;
    const Env v = env_view(tile, s, h, w);
    // per-player and per-env scalars: the global loads are issued first so
    // their latency overlaps the danger map
    float g_py = 0.f, g_px = 0.f;
    int g_alive = 0;
    int64_t g_inv = 0, g_bcap = 0;
    if (lane < P) {
      g_py = st.pos[((size_t)lane * 2 + 0) * N + e];
      g_px = st.pos[((size_t)lane * 2 + 1) * N + e];
      g_alive = st.alive[(size_t)lane * N + e] != 0;
      g_inv = st.invuln[(size_t)lane * N + e];
      g_bcap = st.bombs_cap[(size_t)lane * N + e];
    }
    const int64_t g_t = st.t[e];
    int max_b = 0;
    const int nb = danger_stage_a(v, ds, cfg.fuse_f, cfg.blast, cfg.danger_rounds, &max_b, -1,
                                  ft.weight);
    danger_paint(v, ds, nb, cfg.blast, dng);
    const int live = live_count_of_lane(v, P);
    observe_env<T>(cfg, v, e, pi, dng, live, g_py, g_px, g_alive != 0, g_inv, g_bcap, g_t, ft,
                   obs, danger_out, mm, bm);
  }
}

// ------------------------------------------------------------------ astar

// Per-warp scratch of k_astar: danger, cost, the two fields, own bombs,
// then 32 prefetched per-env scalars (8 bytes each).
__host__ __device__ inline size_t astar_pre_off(int cells) {
  return ((size_t)cells * (4 * 4 + 2) + 15) / 16 * 16 + 64;
}
__host__ __device__ inline size_t astar_warp_bytes(int cells) {
  return astar_pre_off(cells) + 48 * 8;
}

// Prefetch slots of k_astar (one global load per lane, issued before the
// tile staging): the scoring that follows the relaxation is serial on lane
// 0, and without this every scalar it reads would expose a load latency.
// Slots 32..41 keep the candidates' V_opp / V_safe while the hunter's crate
// field reuses the field arrays.
enum {
  AP_TIMER = 0, AP_MODE = 1, AP_NEW_MODE = 2, AP_NEW_TIMER = 3,
  AP_PY = 4, AP_PX = 8, AP_ALIVE = 12,              // + player (QQT_MAX_P slots each)
  AP_CAP = 16, AP_NOISE = 17, AP_MM = 22, AP_BM = 27, AP_BCAP = 28, AP_SPD = 29,
  AP_CAND_OPP = 32, AP_CAND_SAFE = 37
};

// Two multi-source path fields to their common fixed point: row sweeps
// (left->right, right->left) then column sweeps, repeated until no value
// changes.  Values only decrease and every value is a path sum, so any
// sweep order ends at the reference's Jacobi fixed point.
__device__ inline bool relax_two(volatile float* d0, volatile float* d1, const float* cost,
                                 int h, int w, int max_iter) {
  const int lane = lane_id();
  const float INF = __int_as_float(0x7f800000);
  for (int it = 0; it < max_iter; ++it) {
    bool changed = false;
    for (int task = lane; task < 2 * h; task += 32) {
      volatile float* d = task < h ? d0 : d1;
      const int r = task < h ? task : task - h;
      for (int k = 0; k < 2 * w; ++k) {
        const int cc = k < w ? k : 2 * w - 1 - k;
        const int c = r * w + cc;
        const float cst = cost[c];
        if (cst == INF) continue;
        float m = INF;
        if (r > 0) m = fminf(m, d[c - w]);
        if (r < h - 1) m = fminf(m, d[c + w]);
        if (cc > 0) m = fminf(m, d[c - 1]);
        if (cc < w - 1) m = fminf(m, d[c + 1]);
        const float nd = __fadd_rn(m, cst);
        if (nd < d[c]) {
          d[c] = nd;
          changed = true;
        }
      }
    }
    __syncwarp();
    for (int task = lane; task < 2 * w; task += 32) {
      volatile float* d = task < w ? d0 : d1;
      const int cc = task < w ? task : task - w;
      for (int k = 0; k < 2 * h; ++k) {
        const int r = k < h ? k : 2 * h - 1 - k;
        const int c = r * w + cc;
        const float cst = cost[c];
        if (cst == INF) continue;
        float m = INF;
        if (r > 0) m = fminf(m, d[c - w]);
        if (r < h - 1) m = fminf(m, d[c + w]);
        if (cc > 0) m = fminf(m, d[c - 1]);
        if (cc < w - 1) m = fminf(m, d[c + 1]);
        const float nd = __fadd_rn(m, cst);
        if (nd < d[c]) {
          d[c] = nd;
          changed = true;
        }
      }
    }
    __syncwarp();
    if (!__any_sync(QQT_FULL, changed)) return true;
  }
  return false;
}

// The same fixed point with the fields in registers, for boards of H x W
// <= 16 x 16: lane (f, r) = (lane / 16, lane % 16) holds row r of field f
// (f = 0: d0, f = 1: d1) for the row sweeps (left-to-right then
// right-to-left, vertical neighbours by shuffles within the 16-lane half),
// then the rows are transposed through d0 / d1 so that lane (f, c) holds
// column c for the column sweeps.  Every sweep phase relaxes each cell
// against all four neighbours, so a phase that changes nothing is the
// fixed point; the loop stops there.  Returns false if max_phases ran out.
template <int H, int W>
__device__ bool relax_two_reg(float* d0, float* d1, const float* cost, int max_phases,
                              int* phases_out = nullptr) {
  static_assert(H <= 16 && W <= 16, "one row or column per lane of a 16-lane half");
  const int lane = lane_id(), f = lane >> 4, i = lane & 15;
  const float INF = __int_as_float(0x7f800000);
  float* dd = f ? d1 : d0;
  const bool row_lane = i < H, col_lane = i < W;
  float v[W > H ? W : H];                // a row (row phases) or a column (column phases)
  float cr[W];                           // this lane's cost row; columns come from shared memory
#pragma unroll
  for (int c = 0; c < W; ++c) {
    v[c] = row_lane ? dd[i * W + c] : INF;
    cr[c] = row_lane ? cost[i * W + c] : INF;
  }
  bool rows = true, done = false;
  int ph_used = 0;
  for (int ph = 0; ph < max_phases; ++ph) {
    bool ch = false;
    ph_used = ph + 1;
    if (rows) {
      float up[W], dn[W];
#pragma unroll
      for (int c = 0; c < W; ++c) {
        up[c] = __shfl_up_sync(QQT_FULL, v[c], 1, 16);
        dn[c] = __shfl_down_sync(QQT_FULL, v[c], 1, 16);
        if (i == 0) up[c] = INF;
        if (i >= H - 1) dn[c] = INF;
        up[c] = fminf(up[c], dn[c]);
      }
#pragma unroll
      for (int c = 0; c < W; ++c) {
        float m = up[c];
        if (c > 0) m = fminf(m, v[c - 1]);
        if (c < W - 1) m = fminf(m, v[c + 1]);
        const float nd = __fadd_rn(m, cr[c]);
        if (nd < v[c]) { v[c] = nd; ch = true; }
      }
#pragma unroll
      for (int c = W - 1; c >= 0; --c) {
        float m = up[c];
        if (c > 0) m = fminf(m, v[c - 1]);
        if (c < W - 1) m = fminf(m, v[c + 1]);
        const float nd = __fadd_rn(m, cr[c]);
        if (nd < v[c]) { v[c] = nd; ch = true; }
      }
    } else {
      float lf[H], rt[H];
#pragma unroll
      for (int r = 0; r < H; ++r) {
        lf[r] = __shfl_up_sync(QQT_FULL, v[r], 1, 16);
        rt[r] = __shfl_down_sync(QQT_FULL, v[r], 1, 16);
        if (i == 0) lf[r] = INF;
        if (i >= W - 1) rt[r] = INF;
        lf[r] = fminf(lf[r], rt[r]);
      }
      const float* ccol = cost + (col_lane ? i : 0);
#pragma unroll
      for (int r = 0; r < H; ++r) {
        float m = lf[r];
        if (r > 0) m = fminf(m, v[r - 1]);
        if (r < H - 1) m = fminf(m, v[r + 1]);
        const float nd = __fadd_rn(m, col_lane ? ccol[r * W] : INF);
        if (nd < v[r]) { v[r] = nd; ch = true; }
      }
#pragma unroll
      for (int r = H - 1; r >= 0; --r) {
        float m = lf[r];
        if (r > 0) m = fminf(m, v[r - 1]);
        if (r < H - 1) m = fminf(m, v[r + 1]);
        const float nd = __fadd_rn(m, col_lane ? ccol[r * W] : INF);
        if (nd < v[r]) { v[r] = nd; ch = true; }
      }
    }
    done = !__any_sync(QQT_FULL, ch);
    // transpose through the field arrays (also the final write-back)
    if (rows) {
      if (row_lane)
#pragma unroll
        for (int c = 0; c < W; ++c) dd[i * W + c] = v[c];
    } else {
      if (col_lane)
#pragma unroll
        for (int r = 0; r < H; ++r) dd[r * W + i] = v[r];
    }
    __syncwarp();
    if (done) break;
    rows = !rows;
    if (rows) {
#pragma unroll
      for (int c = 0; c < W; ++c) v[c] = row_lane ? dd[i * W + c] : INF;
    } else {
#pragma unroll
      for (int r = 0; r < H; ++r) v[r] = col_lane ? dd[r * W + i] : INF;
    }
    __syncwarp();
  }
  if (phases_out) *phases_out = ph_used;
  return done;
}

// First index of the smallest of five values; the running minimum stays in
// a register (and is returned in *min_out), so the caller's array is only
// indexed by constants and stays in registers too.
__device__ __forceinline__ int argmin5(const float* s, float* min_out = nullptr) {
  int best = 0;
  float bv = s[0];
#pragma unroll
  for (int k = 1; k < 5; ++k)
    if (s[k] < bv) {
      bv = s[k];
      best = k;
    }
  if (min_out) *min_out = bv;
  return best;
}

// EAT: the hunter bot (sim/bots.py:557-561): astar with the crate layer
// (sim/bots.py:376-431) and no mode ticker.
// NP > 0: the player count fixed at compile time; 0: cfg.n_players.
// GS > 0: a GS x GS grid fixed at compile time; 0: the config's grid.
template <bool EAT, int NP = 0, int GS = 0>
__global__ void __launch_bounds__(QQT_NWARP * 32, 3)
k_astar(QqtCfg cfg, QqtState st, const __half* obs, SeatIO io, int pid, const float* noise,
        int64_t* mode_arr, int64_t* timer_arr, int tick16, const int64_t* new_mode,
        const int64_t* new_timer, float* vsafe_out, float* vopp_out, float* vcrate_out,
        const int* cap_max_ptr) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int h = GS > 0 ? GS : cfg.height, w = GS > 0 ? GS : cfg.width, C = h * w;
  const int N = cfg.n_envs, P = NP > 0 ? NP : cfg.n_players;
  const int e0 = blockIdx.x * QQT_TILE_E;
  const float INF = __int_as_float(0x7f800000);
  static_assert(QQT_TILE_E == QQT_NWARP, "one env per warp");
  const int dch = 2 * P + 1;
  // the env's danger channel (fp16 obs row), cells lane + 32 k
  constexpr int kDK = (QQT_MAX_CELLS + 31) / 32;
  float dpre[kDK];
  const bool dpre_ok = C <= 32 * 6;
#pragma unroll
  for (int k = 0; k < kDK; ++k) dpre[k] = 0.f;
  if (dpre_ok && e0 + warp_id() < N) {
    const __half* orow = obs + (size_t)(e0 + warp_id()) * cfg.obs_stride + (size_t)dch * C;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      const int c = lane_id() + 32 * k;
      if (c < C) dpre[k] = __half2float(orow[c]);
    }
  }
  uint64_t pre_v = 0;
  {
    const int e = e0 + warp_id(), l = lane_id();
    if (e < N) {
      if (l == AP_TIMER && mode_arr) pre_v = (uint64_t)timer_arr[e];
      else if (l == AP_MODE && mode_arr) pre_v = (uint64_t)mode_arr[e];
      else if (l == AP_NEW_MODE && mode_arr && tick16) pre_v = (uint64_t)new_mode[e];
      else if (l == AP_NEW_TIMER && mode_arr && tick16) pre_v = (uint64_t)new_timer[e];
      else if (l >= AP_PY && l < AP_PY + P) pre_v = __float_as_uint(st.pos[((size_t)(l - AP_PY) * 2) * N + e]);
      else if (l >= AP_PX && l < AP_PX + P) pre_v = __float_as_uint(st.pos[((size_t)(l - AP_PX) * 2 + 1) * N + e]);
      else if (l >= AP_ALIVE && l < AP_ALIVE + P) pre_v = st.alive[(size_t)(l - AP_ALIVE) * N + e];
      else if (l == AP_CAP) pre_v = (uint64_t)st.blast_cap[(size_t)pid * N + e];
      else if (l >= AP_NOISE && l < AP_NOISE + 5) pre_v = __float_as_uint(noise[(size_t)e * 5 + (l - AP_NOISE)]);
      else if (l >= AP_MM && l < AP_MM + 5) pre_v = io.mm[(size_t)e * io.mm_stride + (l - AP_MM)];
      else if (l == AP_BM) pre_v = io.bm[(size_t)e * io.bm_stride + 1];
      else if (EAT && l == AP_BCAP) pre_v = (uint64_t)st.bombs_cap[(size_t)pid * N + e];
      else if (EAT && l == AP_SPD) pre_v = __float_as_uint(st.spd_g[(size_t)pid * N + e]);
    }
  }
  QQT_PH_START(ph_t0);
  Tile tile = carve_tile(smem, C);
  load_tile(tile, st, N, e0, PL_WALL | PL_BRICK | PL_OWNER | PL_FUSE | (EAT ? PL_CRATE : 0u));
  __syncthreads();
  QQT_PH_AT(3, 0, ph_t0, (blockIdx.x & 3) == 0 && lane_id() == 0);
  QQT_PH(3, 1, (blockIdx.x & 3) == 0 && lane_id() == 0);
  uint8_t* wb = smem + tile_bytes(C) + (size_t)warp_id() * astar_warp_bytes(C);
  uint64_t* pre = (uint64_t*)(wb + astar_pre_off(C));
  pre[lane_id()] = pre_v;
  __syncwarp();
  float* d16 = (float*)wb;
  float* cost = d16 + C;
  float* vs = cost + C;
  float* vo = vs + C;
  uint16_t* own = (uint16_t*)(vo + C);
  const int lane = lane_id();
  // k_astar is launched as k_cap_max's programmatic dependent: everything
  // above reads the step's outputs, complete before k_cap_max started;
  // only the chain-scan length comes from k_cap_max itself
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int cap_max = *cap_max_ptr;
  const int G = cfg.growth_blast_max;

  for (int s = warp_id(); s < QQT_TILE_E; s += QQT_NWARP) {
    const int e = e0 + s;
    if (e >= N) break;
    const Env v = env_view(tile, s, h, w);
    const __half* orow = obs + (size_t)e * cfg.obs_stride + (size_t)dch * C;
#pragma unroll
    for (int k = 0; k < kDK; ++k) {
      const int c = lane + 32 * k;
      if (c >= C) break;
      const float d = dpre_ok ? dpre[k] : __half2float(orow[c]);
      d16[c] = d;
      const bool blk = v.wall[c] || v.brick[c] || v.fuse[c] > 0;
      cost[c] = blk ? INF : __fadd_rn(1.f, __fmul_rn(2.f, d));
      vs[c] = d < 0.35f ? 0.f : INF;
      vo[c] = INF;
    }
    // own live bombs: the threat term (a cell within Manhattan distance G
    // of one, sim/bots.py:301-309) is only read at the five candidates
    const int nown = warp_compact(C, own, [&](int c) { return v.owner[c] == pid && v.fuse[c] > 0; });
    __syncwarp();
    if (lane == 0) {
      for (int o = 0; o < P; ++o) {
        if (o == pid || !pre[AP_ALIVE + o]) continue;
        const int ro = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PY + o])), 0), h - 1);
        const int co = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PX + o])), 0), w - 1);
        vo[ro * w + co] = 0.f;
      }
    }
    __syncwarp();
    QQT_PH(3, 2, (blockIdx.x & 3) == 0 && lane_id() == 0);
    int relax_phases = 0;
    const bool conv = (h == 13 && w == 13)
                          ? relax_two_reg<13, 13>(vs, vo, cost, 2 * (C + 1), &relax_phases)
                          : relax_two(vs, vo, cost, h, w, C + 1);
    QQT_PH(3, 3, (blockIdx.x & 3) == 0 && lane_id() == 0);
    // the phase count of the two-field relaxation, as a stamp id 40 + n
    QQT_PH(3, 40 + min(relax_phases, 200), (blockIdx.x & 3) == 0 && lane_id() == 0);
    if (!conv && lane == 0) flag_error(QQT_DEV_NOT_CONVERGED);
    if (vsafe_out)
      for (int c = lane; c < C; c += 32) vsafe_out[(size_t)e * C + c] = vs[c];
    if (vopp_out)
      for (int c = lane; c < C; c += 32) vopp_out[(size_t)e * C + c] = vo[c];
    bool any_crate = false;
    if (EAT) {
      // keep the candidates' V_opp / V_safe, then relax V_crate (sources =
      // crate cells, same cost and obstacles) in the field arrays
      if (lane < 5) {
        const int r = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PY + pid])), 0), h - 1);
        const int c = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PX + pid])), 0), w - 1);
        const int rr = lane == 0 ? max(r - 1, 0) : (lane == 1 ? min(r + 1, h - 1) : r);
        const int cc = lane == 2 ? max(c - 1, 0) : (lane == 3 ? min(c + 1, w - 1) : c);
        pre[AP_CAND_OPP + lane] = __float_as_uint(vo[rr * w + cc]);
        pre[AP_CAND_SAFE + lane] = __float_as_uint(vs[rr * w + cc]);
      }
      bool mine = false;
      __syncwarp();
      for (int c = lane; c < C; c += 32) {
        const bool cr = v.crate[c] != 0;
        mine |= cr;
        vs[c] = cr ? 0.f : INF;
        vo[c] = INF;
      }
      any_crate = __any_sync(QQT_FULL, mine);
      __syncwarp();
      const bool conv2 = (h == 13 && w == 13) ? relax_two_reg<13, 13>(vs, vo, cost, 2 * (C + 1))
                                              : relax_two(vs, vo, cost, h, w, C + 1);
      if (!conv2 && lane == 0) flag_error(QQT_DEV_NOT_CONVERGED);
      if (vcrate_out)
        for (int c = lane; c < C; c += 32) vcrate_out[(size_t)e * C + c] = vs[c];
    }

    // scoring (sim/bots.py:433-508): candidate k (up, down, left, right,
    // idle) on lane k, each with the same float operations as a serial
    // loop; lane 0 combines the five.  Lanes 5..31 repeat the idle
    // candidate and are left out of every vote.
    int mode = 0;
    const bool has_mode = mode_arr != nullptr;
    if (has_mode) {
      int64_t tm = (int64_t)pre[AP_TIMER] - 1;
      int64_t md = (int64_t)pre[AP_MODE];
      if (tick16 && tm <= 0) {
        md = (int64_t)pre[AP_NEW_MODE];
        tm = (int64_t)pre[AP_NEW_TIMER];
      }
      if (lane == 0) {
        timer_arr[e] = tm;
        mode_arr[e] = md;
      }
      mode = (int)md;
    }
    const float py = __uint_as_float((uint32_t)pre[AP_PY + pid]);
    const float px = __uint_as_float((uint32_t)pre[AP_PX + pid]);
    const int r = min(max((int)floorf(py), 0), h - 1), c = min(max((int)floorf(px), 0), w - 1);
    const float own_dng = d16[r * w + c];
    const bool cand = lane < 5;
    const int k = cand ? lane : 4;
    const int rk = k == 0 ? max(r - 1, 0) : (k == 1 ? min(r + 1, h - 1) : r);
    const int ck = k == 2 ? max(c - 1, 0) : (k == 3 ? min(c + 1, w - 1) : c);
    const int q = rk * w + ck;
    float vopp_k, vsafe_k, vcrate_k;
    if (EAT) {
      vopp_k = __uint_as_float((uint32_t)pre[AP_CAND_OPP + k]);
      vsafe_k = __uint_as_float((uint32_t)pre[AP_CAND_SAFE + k]);
      vcrate_k = vs[q];
    } else {
      vopp_k = vo[q];
      vsafe_k = vs[q];
      vcrate_k = INF;
    }
    const float dng_k = d16[q];
    bool thr = false;
    for (int i = 0; i < nown && !thr; ++i) {
      const int b = own[i], br = b / w, bc = b - br * w;
      if (abs(br - rk) + abs(bc - ck) <= G) thr = true;
    }
    const float thr_k = thr ? 1.f : 0.f;
    const bool legal_k = pre[AP_MM + k] && !(v.wall[q] || v.brick[q]);
    const float nz_k = __fmul_rn(0.05f, __uint_as_float((uint32_t)pre[AP_NOISE + k]));
    float app = __fadd_rn(__fadd_rn(__fadd_rn(vopp_k, __fmul_rn(2.f, dng_k)), __fmul_rn(2.f, thr_k)),
                          nz_k);
    if (dng_k >= 0.5f || !legal_k) app = INF;
    const bool app_ok = __any_sync(QQT_FULL, cand && app < INF);
    const bool use_esc = own_dng >= 0.35f || !app_ok;
    float esc = __fadd_rn(__fadd_rn(__fmul_rn(vsafe_k, 100.f), __fmul_rn(2.f, thr_k)), nz_k);
    if ((use_esc && k == 4) || !legal_k) esc = INF;
    if (EAT) {
      // crate layer: >= 2 of the growth attributes under 70 % of their
      // caps, a crate on the board, alive -> descend V_crate (no idling
      // when a move is better), unless no crate is reachable
      const float fb = __fdiv_rn((float)(int64_t)pre[AP_BCAP], (float)cfg.growth_bombs_max);
      const float fz = __fdiv_rn((float)(int64_t)pre[AP_CAP], (float)cfg.growth_blast_max);
      const float fs = __fdiv_rn(__uint_as_float((uint32_t)pre[AP_SPD]), cfg.growth_speed_max);
      const int low = (fb < 0.7f) + (fz < 0.7f) + (fs < 0.7f);
      bool eat_on = low >= 2 && any_crate && pre[AP_ALIVE + pid] != 0;
      float eat = __fadd_rn(__fadd_rn(__fmul_rn(vcrate_k, 100.f), __fmul_rn(2.f, dng_k)), nz_k);
      if (dng_k >= 0.5f || !legal_k) eat = INF;
      const float no_idle = fminf(fminf(__shfl_sync(QQT_FULL, eat, 0), __shfl_sync(QQT_FULL, eat, 1)),
                                  fminf(__shfl_sync(QQT_FULL, eat, 2), __shfl_sync(QQT_FULL, eat, 3)));
      if (k == 4 && no_idle < eat) eat = INF;
      eat_on = eat_on && fminf(no_idle, __shfl_sync(QQT_FULL, eat, 4)) < INF;
      if (eat_on) app = eat;
    }
    float score = use_esc ? esc : app;
    if (has_mode && mode == 1) {
      float f = __fadd_rn(__fadd_rn(__fadd_rn(-fminf(vopp_k, 1e3f), __fmul_rn(2.f, dng_k)),
                                    __fmul_rn(2.f, thr_k)), nz_k);
      if (dng_k >= 0.5f || !legal_k) f = INF;
      score = use_esc ? esc : f;
    }
    const unsigned legal_m = __ballot_sync(QQT_FULL, cand && legal_k);
    const unsigned safe_m =
        __ballot_sync(QQT_FULL, cand && legal_k && dng_k < 0.35f && thr_k == 0.f);
    float sc[5], dl[5];
#pragma unroll
    for (int j = 0; j < 5; ++j) {
      sc[j] = __shfl_sync(QQT_FULL, score, j);
      dl[j] = __shfl_sync(QQT_FULL, legal_k ? dng_k : INF, j);
    }
    // chain term: a live bomb with fuse 1..10 within cap_max cells in a
    // straight line (the batch's largest blast cap, sim/bots.py:484), one
    // (distance, direction) probe per lane
    const int cap = (int)(int64_t)pre[AP_CAP];
    bool chain = false;
    for (int base = 0; base < 4 * cap_max && !chain; base += 32) {
      const int j = base + lane;
      bool hit = false;
      if (j < 4 * cap_max) {
        const int dist = (j >> 2) + 1, d = j & 3;
        const int r2 = r + (d == 0 ? -dist : (d == 1 ? dist : 0));
        const int c2 = c + (d == 2 ? -dist : (d == 3 ? dist : 0));
        if (r2 >= 0 && r2 < h && c2 >= 0 && c2 < w) {
          const int f = v.fuse[r2 * w + c2];
          hit = f > 0 && f <= 10;
        }
      }
      chain = __any_sync(QQT_FULL, hit);
    }
    if (lane == 0) {
      int move = argmin5(sc);
      bool finite = false;
      float dmv[5];
#pragma unroll
      for (int j = 0; j < 5; ++j) {
        finite |= sc[j] < INF;
        dmv[j] = j < 4 ? dl[j] : INF;
      }
      if (!finite && legal_m != 0) {
        float fmin;
        const int fm = argmin5(dmv, &fmin);
        move = fmin < INF ? fm : argmin5(dl);
      }
      long long dr_o = 1000000000LL, dc_o = 1000000000LL;
      for (int o = 0; o < P; ++o) {
        if (o == pid || !pre[AP_ALIVE + o]) continue;
        const int ro = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PY + o])), 0), h - 1);
        const int co = min(max((int)floorf(__uint_as_float((uint32_t)pre[AP_PX + o])), 0), w - 1);
        dr_o = llabs((long long)(r - ro));
        dc_o = llabs((long long)(c - co));
      }
      const bool aligned = (dr_o == 0 && dc_o <= cap) || (dc_o == 0 && dr_o <= cap);
      const long long manh = min(dr_o + dc_o, 100000000LL);
      const bool near = manh <= max((long long)cap + 1, 1LL);
      const bool can = pre[AP_BM] != 0;
      const bool can_escape = safe_m != 0;
      bool place = can && (aligned || near || chain) && own_dng < 0.2f && can_escape;
      if (has_mode && mode == 1) place = can && (aligned || near) && own_dng < 0.2f && can_escape;
      const bool alive = pre[AP_ALIVE + pid] != 0;
      io.act[(size_t)e * io.act_stride + 0] = alive ? move : 4;
      io.act[(size_t)e * io.act_stride + 1] = alive ? (place ? 1 : 0) : 0;
    }
    __syncwarp();
    QQT_PH(3, 4, (blockIdx.x & 3) == 0 && lane_id() == 0);
  }
}

// One block: the maximum over the seat's blast caps (0 for an empty batch),
// written once, so no memset precedes it and the bot's first node in a
// captured tick is a kernel.
__global__ void __launch_bounds__(1024) k_cap_max(const int64_t* blast_cap, int n, int* out) {
  // the bot kernel after it may start staging now (it waits for this
  // kernel's result before reading it)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int wmax[32];
  int m = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = max(m, (int)blast_cap[i]);
  m = warp_max(m);
  if (lane_id() == 0) wmax[warp_id()] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0;
    m = warp_max(m);
    if (threadIdx.x == 0) *out = m;
  }
}

// ---------------------------------------------------------- random / greedy

__device__ __forceinline__ int sample_legal(const uint8_t* mask, int k, float u) {
  float cs[5];
  float acc = 0.f;
  for (int i = 0; i < k; ++i) {
    acc = __fadd_rn(acc, mask[i] ? 1.f : 0.f);
    cs[i] = acc;
  }
  const float us = __fmul_rn(u, fmaxf(cs[k - 1], 1e-6f));
  int a = 0;
  for (int i = 0; i < k; ++i) a += us > cs[i];
  return a;
}

__global__ void k_random(int n, const uint8_t* alive, SeatIO io, int pid, const float* u_move,
                         const float* u_bomb, float rate) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const bool al = alive[(size_t)pid * n + e] != 0;
  const int move = sample_legal(io.mm + (size_t)e * io.mm_stride, 5, u_move[e]);
  const bool bomb = u_bomb[e] < rate && io.bm[(size_t)e * io.bm_stride + 1];
  io.act[(size_t)e * io.act_stride + 0] = al ? move : 4;
  io.act[(size_t)e * io.act_stride + 1] = (al && bomb) ? 1 : 0;
}

__global__ void k_greedy(QqtCfg cfg, QqtState st, const __half* obs, SeatIO io, int pid,
                         const float* noise) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const int N = cfg.n_envs, P = cfg.n_players, h = cfg.height, w = cfg.width, C = h * w;
  if (e >= N) return;
  const float INF = __int_as_float(0x7f800000);
  const __half* drow = obs + (size_t)e * cfg.obs_stride + (size_t)(2 * P + 1) * C;
  const int r = min(max((int)floorf(st.pos[((size_t)pid * 2) * N + e]), 0), h - 1);
  const int c = min(max((int)floorf(st.pos[((size_t)pid * 2 + 1) * N + e]), 0), w - 1);
  const float own = __half2float(drow[r * w + c]);
  const int cr[5] = {max(r - 1, 0), min(r + 1, h - 1), r, r, r};
  const int ccs[5] = {c, c, max(c - 1, 0), min(c + 1, w - 1), c};
  float dist[5], dng[5];
  bool blk[5];
  for (int k = 0; k < 5; ++k) {
    const int q = cr[k] * w + ccs[k];
    dng[k] = __half2float(drow[q]);
    blk[k] = st.wall[(size_t)e * C + q] || st.brick[(size_t)e * C + q];
    dist[k] = 1e9f;
  }
  for (int o = 0; o < P; ++o) {
    if (o == pid) continue;
    const int ro = min(max((int)floorf(st.pos[((size_t)o * 2) * N + e]), 0), h - 1);
    const int co = min(max((int)floorf(st.pos[((size_t)o * 2 + 1) * N + e]), 0), w - 1);
    const bool al = st.alive[(size_t)o * N + e] != 0;
    for (int k = 0; k < 5; ++k) {
      const float d = al ? (float)max(abs(cr[k] - ro), abs(ccs[k] - co)) : 1e9f;
      dist[k] = fminf(dist[k], d);
    }
  }
  const uint8_t* mrow = io.mm + (size_t)e * io.mm_stride;
  int best = 0, esc_d = 0;
  // best_dng = dng[best] without a run-time index into dng
  float best_s = INF, esc_s = INF, best_dng = dng[0];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const bool legal = mrow[k] && !blk[k];
    const float nz = __fmul_rn(0.05f, noise[(size_t)e * 5 + k]);
    const float sc = legal ? __fadd_rn(__fadd_rn(dist[k], __fmul_rn(2.f, dng[k])), nz) : INF;
    if (sc < best_s) {
      best_s = sc;
      best = k;
      best_dng = dng[k];
    }
    const float es = legal ? dng[k] : INF;
    if (es < esc_s) {
      esc_s = es;
      esc_d = k;
    }
  }
  const bool use_safe = best_s < INF && best_dng < 0.35f;
  const int move = use_safe ? best : esc_d;
  const bool place = io.bm[(size_t)e * io.bm_stride + 1] &&
                     dist[4] < (float)st.blast_cap[(size_t)pid * N + e] && own < 0.2f;
  const bool al = st.alive[(size_t)pid * N + e] != 0;
  io.act[(size_t)e * io.act_stride + 0] = al ? move : 4;
  io.act[(size_t)e * io.act_stride + 1] = (al && place) ? 1 : 0;
}

}  // namespace qqt

using namespace qqt;

// ------------------------------------------------ LSTM local-view features

__device__ __forceinline__ float from_obs(float v) { return v; }
__device__ __forceinline__ float from_obs(__half v) { return __half2float(v); }

// Per-player features of the LSTM policy from the shared observation rows
// (sim/obs.py:241-340); one warp per (env, output player m):
//   local [m] the 7x7 window of every channel centred on the player's cell,
//             the reference's zero padding of 3 and coordinate clamp
//   rel   [m] opponents (m + i + 1) % P: [row delta, column delta, alive];
//             then the k = min(10 - (P-1), H*W) cells nearest to the player
//             (L1, a non-bomb cell counting 1e6) by k warp-argmin rounds
//             over 64-bit keys (distance, flat cell), written as [column
//             delta, row delta, 0, is-bomb]
//   glob  [m] dtype(t) / max_steps, dtype(hp) / max_hp, danger under the
//             player, live bombs / max_bombs, sum(fuse) / (max_bombs * fuse)
// The reference orders equal distances by torch.topk, which leaves that
// order open; here it is ascending flat cell index.
template <typename T>
__global__ void k_local_view(QqtCfg cfg, QqtState st, const T* __restrict__ obs, int max_bombs,
                             int po, T* __restrict__ local, T* __restrict__ rel,
                             T* __restrict__ glob) {
  const int gw = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
  const int lane = lane_id();
  const int N = cfg.n_envs, P = cfg.n_players, H = cfg.height, W = cfg.width, C = H * W;
  const int CH = cfg.obs_channels;
  if (gw >= N * po) return;
  const int e = gw / po, m = gw - e * po;
  const float py = st.pos[(size_t)(2 * m) * N + e], px = st.pos[(size_t)(2 * m + 1) * N + e];
  const int cy = (int)floorf(py), cx = (int)floorf(px);
  const T* orow = obs + (size_t)e * cfg.obs_stride;
  T* lo = local + ((size_t)e * po + m) * CH * 49;
  const int total = CH * 49;
  for (int base = 0; base < total; base += 8 * 32) {
    T vals[8];                            // eight independent loads in flight per lane
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * 32 + lane;
      vals[u] = to_obs<T>(0.f);
      if (i < total) {
        const int ch = i / 49, k = i - ch * 49, dy = k / 7, dx = k - dy * 7;
        const int ys = min(max(cy + dy, 0), H + 5) - 3, xs = min(max(cx + dx, 0), W + 5) - 3;
        if (ys >= 0 && ys < H && xs >= 0 && xs < W) vals[u] = orow[(size_t)ch * C + ys * W + xs];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * 32 + lane;
      if (i < total) lo[i] = vals[u];
    }
  }
  T* re = rel + ((size_t)e * po + m) * 60;
  for (int i = lane; i < 60; i += 32) re[i] = to_obs<T>(0.f);
  __syncwarp();
  const int n_opp = P - 1;
  if (lane < n_opp) {
    const int opp = (m + lane + 1) % P;
    re[lane * 6 + 0] = to_obs<T>(__fsub_rn(st.pos[(size_t)(2 * opp) * N + e], py));
    re[lane * 6 + 1] = to_obs<T>(__fsub_rn(st.pos[(size_t)(2 * opp + 1) * N + e], px));
    re[lane * 6 + 2] = to_obs<T>(st.alive[(size_t)opp * N + e] ? 1.f : 0.f);
  }
  // nearest cells: each lane owns cells lane, lane + 32, ... (at most 14),
  // their distance keys held in registers (a non-bomb cell counts 1e6; a cell
  // past the grid or already taken counts 2^32 - 1)
  constexpr int kOwn = (QQT_MAX_CELLS + 31) / 32;
  const int16_t* frow = st.fuse + (size_t)e * C;
  int nb = 0, fsum = 0;
  unsigned dk[kOwn];
#pragma unroll
  for (int j = 0; j < kOwn; ++j) {
    const int c = lane + 32 * j;
    unsigned d = 0xffffffffu;
    if (c < C) {
      const int f = frow[c];
      nb += f > 0;
      fsum += f;
      const int r = c / W, q = c - r * W;
      d = f > 0 ? (unsigned)(abs(r - cy) + abs(q - cx)) : 1000000u;
    }
    dk[j] = d;
  }
  nb = __reduce_add_sync(QQT_FULL, nb);
  fsum = __reduce_add_sync(QQT_FULL, fsum);
  const int k = min(10 - n_opp, C);
  for (int j = 0; j < k; ++j) {
    unsigned long long best = ~0ull;
#pragma unroll
    for (int jj = 0; jj < kOwn; ++jj) {
      const unsigned long long key =
          ((unsigned long long)dk[jj] << 32) | (unsigned)(lane + 32 * jj);
      best = key < best ? key : best;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(QQT_FULL, best, o);
      best = other < best ? other : best;
    }
    const int c = (int)(best & 0xffffffffull);
#pragma unroll
    for (int jj = 0; jj < kOwn; ++jj)
      if (lane == (c & 31) && jj == (c >> 5)) dk[jj] = 0xffffffffu;
    if (lane == 0) {
      const int r = c / W, q = c - r * W;
      T* sl = re + (n_opp + j) * 6;
      sl[0] = to_obs<T>(__fsub_rn((float)q, (float)cx));
      sl[1] = to_obs<T>(__fsub_rn((float)r, (float)cy));
      sl[3] = to_obs<T>((best >> 32) < 100000ull ? 1.f : 0.f);
    }
  }
  if (lane == 0) {
    T* gl = glob + ((size_t)e * po + m) * 5;
    const float tq = from_obs(to_obs<T>((float)st.t[e]));
    const float hq = from_obs(to_obs<T>((float)st.hp[(size_t)m * N + e]));
    gl[0] = to_obs<T>(__fdiv_rn(tq, (float)cfg.max_steps));
    gl[1] = to_obs<T>(__fdiv_rn(hq, (float)cfg.max_hp));
    const bool in = cy >= 0 && cy < H && cx >= 0 && cx < W;
    gl[2] = in ? orow[(size_t)(2 * P + 1) * C + cy * W + cx] : to_obs<T>(0.f);
    gl[3] = to_obs<T>(__fdiv_rn((float)nb, (float)max_bombs));
    gl[4] = to_obs<T>(__fdiv_rn((float)fsum, (float)(max_bombs * cfg.fuse)));
  }
}

extern "C" int qqt_local_view(const QqtCfg* cfg, const QqtState* st, const void* obs,
                              int32_t max_bombs, int32_t only_p0, void* local, void* rel,
                              void* glob, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if (!st || !obs || !local || !rel || !glob || max_bombs <= 0) return QQT_E_ARG;
  if (cfg->obs_channels < 2 * cfg->n_players + 2 ||
      cfg->obs_stride < cfg->obs_channels * cfg->height * cfg->width)
    return QQT_E_ARG;
  const int po = only_p0 ? 1 : cfg->n_players;
  const int64_t warps = (int64_t)cfg->n_envs * po;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  if (cfg->obs_fp32)
    k_local_view<float><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        *cfg, *st, (const float*)obs, max_bombs, po, (float*)local, (float*)rel, (float*)glob);
  else
    k_local_view<__half><<<blocks, 256, 0, (cudaStream_t)stream>>>(
        *cfg, *st, (const __half*)obs, max_bombs, po, (__half*)local, (__half*)rel,
        (__half*)glob);
  return launch_status();
}

extern "C" int qqt_observe(const QqtCfg* cfg, const QqtState* st, void* obs, float* danger,
                           uint8_t* mm, uint8_t* bm, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if (!st) return QQT_E_ARG;
  const int C = cfg->height * cfg->width;
  if (obs) {
    const int epc = cfg->obs_fp32 ? 4 : 8;
    if (cfg->obs_stride % epc || cfg->obs_stride < cfg->obs_channels * C) return QQT_E_ALIGN;
    if (((uintptr_t)obs) & 15) return QQT_E_ALIGN;
  }
  const size_t sm = tile_bytes(C) + QQT_NWARP * obs_layout(C).total;
  const int blocks = (cfg->n_envs + QQT_TILE_E - 1) / QQT_TILE_E;
  if (cfg->obs_fp32) {
    cudaFuncSetAttribute(k_observe<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k_observe<true><<<blocks, QQT_NWARP * 32, sm, (cudaStream_t)stream>>>(*cfg, *st, obs, danger, mm, bm);
  } else {
    cudaFuncSetAttribute(k_observe<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k_observe<false><<<blocks, QQT_NWARP * 32, sm, (cudaStream_t)stream>>>(*cfg, *st, obs, danger, mm, bm);
  }
  return launch_status();
}

extern "C" int qqt_legal_mask(const QqtCfg* cfg, const QqtState* st, uint8_t* mm, uint8_t* bm,
                              qqt_stream_t stream) {
  if (!mm || !bm) return QQT_E_ARG;
  return qqt_observe(cfg, st, nullptr, nullptr, mm, bm, stream);
}

static int seat_io(const uint8_t* mm, int32_t mm_stride, const uint8_t* bm, int32_t bm_stride,
                   int64_t* act, int32_t act_stride, SeatIO* io) {
  if (!mm || !bm || !act || mm_stride < 5 || bm_stride < 2 || act_stride < 2) return QQT_E_ARG;
  io->mm = mm;
  io->bm = bm;
  io->act = act;
  io->mm_stride = mm_stride;
  io->bm_stride = bm_stride;
  io->act_stride = act_stride;
  return QQT_OK;
}

template <bool EAT>
static int launch_astar(const QqtCfg* cfg, const QqtState* st, const void* obs,
                        const uint8_t* mm, int32_t mm_stride, const uint8_t* bm,
                        int32_t bm_stride, int32_t pid, const float* noise, int64_t* mode,
                        int64_t* timer, int32_t tick16, const int64_t* new_mode,
                        const int64_t* new_timer, int64_t* act, int32_t act_stride,
                        float* vsafe, float* vopp, float* vcrate, void* scratch,
                        qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  SeatIO io;
  if ((rc = seat_io(mm, mm_stride, bm, bm_stride, act, act_stride, &io))) return rc;
  if (!st || !obs || !noise || !scratch) return QQT_E_ARG;
  if (pid < 0 || pid >= cfg->n_players || cfg->obs_fp32) return QQT_E_ARG;
  if ((mode == nullptr) != (timer == nullptr)) return QQT_E_ARG;
  if (mode && tick16 && (!new_mode || !new_timer)) return QQT_E_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int N = cfg->n_envs, C = cfg->height * cfg->width;
  int* capmax = (int*)scratch;
  k_cap_max<<<1, 1024, 0, s>>>(st->blast_cap + (size_t)pid * N, N, capmax);
  const size_t sm = tile_bytes(C) + QQT_NWARP * astar_warp_bytes(C);
  const bool two = cfg->n_players == 2, g13 = cfg->height == 13 && cfg->width == 13;
  auto kern = two ? (g13 ? k_astar<EAT, 2, 13> : k_astar<EAT, 2>) : k_astar<EAT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)((N + QQT_TILE_E - 1) / QQT_TILE_E), 1, 1);
  lc.blockDim = dim3(QQT_NWARP * 32, 1, 1);
  lc.dynamicSmemBytes = sm;
  lc.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  if (cudaLaunchKernelEx(&lc, kern, *cfg, *st, (const __half*)obs, io, pid, noise, mode, timer,
                         tick16, new_mode, new_timer, vsafe, vopp, vcrate,
                         (const int*)capmax) != cudaSuccess)
    return QQT_E_LAUNCH;
  return launch_status();
}

extern "C" int qqt_astar_act(const QqtCfg* cfg, const QqtState* st, const void* obs,
                             const uint8_t* mm, int32_t mm_stride, const uint8_t* bm,
                             int32_t bm_stride, int32_t pid, const float* noise, int64_t* mode,
                             int64_t* timer, int32_t tick16, const int64_t* new_mode,
                             const int64_t* new_timer, int64_t* act, int32_t act_stride,
                             float* vsafe, float* vopp, void* scratch, qqt_stream_t stream) {
  return launch_astar<false>(cfg, st, obs, mm, mm_stride, bm, bm_stride, pid, noise, mode, timer,
                             tick16, new_mode, new_timer, act, act_stride, vsafe, vopp, nullptr,
                             scratch, stream);
}

extern "C" int qqt_hunter_act(const QqtCfg* cfg, const QqtState* st, const void* obs,
                              const uint8_t* mm, int32_t mm_stride, const uint8_t* bm,
                              int32_t bm_stride, int32_t pid, const float* noise, int64_t* act,
                              int32_t act_stride, float* vsafe, float* vopp, float* vcrate,
                              void* scratch, qqt_stream_t stream) {
  return launch_astar<true>(cfg, st, obs, mm, mm_stride, bm, bm_stride, pid, noise, nullptr,
                            nullptr, 0, nullptr, nullptr, act, act_stride, vsafe, vopp, vcrate,
                            scratch, stream);
}

extern "C" int qqt_random_act(const QqtCfg* cfg, const QqtState* st, const uint8_t* mm,
                              int32_t mm_stride, const uint8_t* bm, int32_t bm_stride, int32_t pid,
                              const float* u_move, const float* u_bomb, float bomb_rate,
                              int64_t* act, int32_t act_stride, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  SeatIO io;
  if ((rc = seat_io(mm, mm_stride, bm, bm_stride, act, act_stride, &io))) return rc;
  if (!st || !u_move || !u_bomb || pid < 0 || pid >= cfg->n_players) return QQT_E_ARG;
  const int N = cfg->n_envs;
  k_random<<<(N + 127) / 128, 128, 0, (cudaStream_t)stream>>>(N, st->alive, io, pid, u_move, u_bomb,
                                                                bomb_rate);
  return launch_status();
}

extern "C" int qqt_greedy_act(const QqtCfg* cfg, const QqtState* st, const void* obs,
                              const uint8_t* mm, int32_t mm_stride, const uint8_t* bm,
                              int32_t bm_stride, int32_t pid, const float* noise, int64_t* act,
                              int32_t act_stride, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  SeatIO io;
  if ((rc = seat_io(mm, mm_stride, bm, bm_stride, act, act_stride, &io))) return rc;
  if (!st || !obs || !noise || pid < 0 || pid >= cfg->n_players || cfg->obs_fp32)
    return QQT_E_ARG;
  const int N = cfg->n_envs;
  k_greedy<<<(N + 127) / 128, 128, 0, (cudaStream_t)stream>>>(*cfg, *st, (const __half*)obs, io, pid,
                                                                noise);
  return launch_status();
}

extern "C" int qqt_get_error(uint32_t* code_out) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, qqt::g_error, sizeof(v)) != cudaSuccess) return QQT_E_LAUNCH;
  const unsigned z = 0;
  if (cudaMemcpyToSymbol(qqt::g_error, &z, sizeof(z)) != cudaSuccess) return QQT_E_LAUNCH;
  if (code_out) *code_out = v;
  return QQT_OK;
}

extern "C" const char* qqt_version(void) { return "qqt_b200 0.1 sm_100a"; }
