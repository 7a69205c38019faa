// Device auto-reset with per-episode level generation (replaces the host
// side of BatchedSim.reset_, sim/torch_sim.py:178-420, and the level
// generators of sim/mapgen.py).
//
// One warp per env; a warp whose env did not end leaves at once.  The new
// level is built cell-parallel (lanes over cells) into the warp's shared
// scratch, written out, and -- when the caller passes observation rows --
// observed for the new episode with the same routine as the step's fused
// observation.  Every random quantity is a counter-based draw: the 24-bit
// SplitMix64 finaliser of (seed ^ env << 32 ^ episode ^ family << 56) +
// index, as a uniform k / 2^24 or as an integer low + (k * range) >> 24.
// The level rules and their float32 arithmetic are the reference's:
//   kind      r < pure_open | < +open_fraction | < +ring_fraction | corridor
//   corridor  top rows t ~ U{0..T} (or fixed T), walls on rows < t and the
//             last T - t rows; side bricks on rows >= t; edge segments of
//             length 2 + floor(3u) from floor(u * span + t) when u < density;
//             a horizontal segment on rows t, t + 1; spawn cells and their
//             4-neighbours cleared of walls and bricks
//   open      0..obst_max single walls on the cells with the smallest keys,
//             spawn neighbourhoods cleared (none on pure-open maps)
//   ring      the central block of walls, band bricks where u < density,
//             ring spawn neighbourhoods cleared

#include "qqt_common.cuh"

namespace qqt {

enum { MG_KIND = 1, MG_OBST_N, MG_OBST_KEY, MG_RING, MG_TOP, MG_VSEG, MG_HSEG, MG_HAZARD };

__device__ __forceinline__ uint64_t mg_key(const QqtMapGen& g, int e, int64_t ep, int fam) {
  return g.seed ^ ((uint64_t)e << 32) ^ (uint64_t)ep ^ ((uint64_t)fam << 56);
}
__device__ __forceinline__ float mg_u(const QqtMapGen& g, int e, int64_t ep, int fam, int i) {
  return hash_uniform(mg_key(g, e, ep, fam) + (uint64_t)i);
}
__device__ __forceinline__ uint32_t mg_u24(const QqtMapGen& g, int e, int64_t ep, int fam,
                                           int i) {
  return hash_u24(mg_key(g, e, ep, fam) + (uint64_t)i);
}
__device__ __forceinline__ bool mg_bit(const uint32_t* words, int c) {
  return (words[c >> 5] >> (c & 31)) & 1u;
}

// Per-warp scratch (16-byte aligned sections): the new level's planes (4 u8
// planes and owner, then the two i16 planes), a zero danger map, the player
// info of the observation.
__host__ __device__ inline size_t reset_i16_off(int cells) {
  return ((size_t)cells * 5 + 1) & ~(size_t)1;
}
__host__ __device__ inline size_t reset_dng_off(int cells) {
  return (reset_i16_off(cells) + (size_t)cells * 4 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t reset_pinfo_off(int cells) {
  return (reset_dng_off(cells) + (size_t)cells * 4 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t reset_warp_bytes(int cells) {
  return (reset_pinfo_off(cells) + QQT_MAX_P * sizeof(PInfo) + 15) & ~(size_t)15;
}

template <bool OBS>
__global__ void __launch_bounds__(QQT_NWARP * 32)
k_map_reset(QqtCfg cfg, QqtState st, QqtMapGen g, const uint8_t* __restrict__ done,
            __half* obs, uint8_t* mm, uint8_t* bm, uint32_t* obs_tiles) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ FuseTables ft;
  const int e = blockIdx.x * QQT_NWARP + warp_id();
  const int N = cfg.n_envs, h = cfg.height, w = cfg.width, C = h * w, P = cfg.n_players;
  const int lane = lane_id();
  if (e >= N || !done[e]) return;          // warp-uniform
  if (OBS) {
    // every active warp writes the same table values, then reads its own
    if (lane < 32) {
      ft.weight[lane] = fuse_weight(lane, cfg.fuse_f);
      ft.norm[lane] = __fdiv_rn((float)lane, cfg.fuse_f);
      ft.capv[lane] = __fdiv_rn((float)lane, cfg.obs_growth_bombs_max);
    }
  }
  uint8_t* wb = smem + (size_t)warp_id() * reset_warp_bytes(C);
  Env v;
  v.wall = wb;
  v.brick = wb + C;
  v.crate = wb + 2 * C;
  v.recycle = wb + 3 * C;
  v.owner = (int8_t*)(wb + 4 * C);
  v.fuse = (int16_t*)(wb + reset_i16_off(C));
  v.blast = v.fuse + C;
  v.h = h;
  v.w = w;
  v.cells = C;
  float* dng = (float*)(wb + reset_dng_off(C));
  PInfo* pinfo = (PInfo*)(wb + reset_pinfo_off(C));

  const int64_t ep = g.episode[e];
  // ---- level kind (sim/torch_sim.py:249-258); 3 = open-mode map
  int kind = 3;
  bool pure = false;
  if (g.corridor_mode) {
    const float r = mg_u(g, e, ep, MG_KIND, 0);
    pure = r < g.cut_pure;
    kind = r < g.cut_open ? 1 : (r < g.cut_ring ? 2 : 0);
  }
  // ---- corridor draws (sim/mapgen.py:15-62, 98-194)
  const int T = g.top_wall_rows;
  const int top = g.random_wall_rows
                      ? (int)(((uint64_t)mg_u24(g, e, ep, MG_TOP, 0) * (uint64_t)(T + 1)) >> 24)
                      : T;
  const int bot = g.random_wall_rows ? T - top : 0;
  int vs[4] = {0, 0, 0, 0}, ve[4] = {0, 0, 0, 0};
  int hs = 0, he = 0;
  bool hon = false;
  if (kind == 0 && g.wall_density > 0.f) {
    const float span = g.random_wall_rows ? (float)max(h - bot - 4 - top, 1) : (float)(h - T - 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= g.n_edge) break;
      const int s = (int)__fadd_rn(__fmul_rn(mg_u(g, e, ep, MG_VSEG, 3 * i), span), (float)top);
      const int ln = 2 + (int)__fmul_rn(mg_u(g, e, ep, MG_VSEG, 3 * i + 1), 3.f);
      if (mg_u(g, e, ep, MG_VSEG, 3 * i + 2) < g.wall_density) {
        vs[i] = s;
        ve[i] = s + ln;
      }
    }
    if (g.corr_c1 - g.corr_c0 > 4) {
      hs = (int)__fadd_rn(__fmul_rn(mg_u(g, e, ep, MG_HSEG, 0), (float)(g.corr_c1 - g.corr_c0 - 4)),
                          (float)g.corr_c0);
      he = hs + 2 + (int)__fmul_rn(mg_u(g, e, ep, MG_HSEG, 1), 3.f);
      hon = mg_u(g, e, ep, MG_HSEG, 2) < g.wall_density;
    }
  }
  const int band_lo = top, band_hi = g.random_wall_rows ? top + 2 : top + min(2, h - T);
  // ---- cells: walls and bricks of every kind but the open obstacles
  for (int c = lane; c < C; c += 32) {
    const int row = c / w, col = c - row * w;
    bool wl = false, br = false;
    if (kind == 0) {
      wl = (row < top || row >= h - bot) && !mg_bit(g.clear_spawn, c);
      br = (col < g.corr_c0 || col >= g.corr_c1) && row >= top;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i < g.n_edge && col == g.edge_cols[i] && row >= vs[i] && row < ve[i]) br = true;
      if (hon && row >= band_lo && row < band_hi && col >= g.corr_c0 && col < g.corr_c1 &&
          col >= hs && col < he)
        br = true;
      br = br && !mg_bit(g.clear_spawn, c);
    } else if (kind == 2) {
      const bool in_blk = row >= g.ring_r0 && row < g.ring_r1 && col >= g.ring_c0 && col < g.ring_c1;
      const bool in_ext = row >= g.ring_r0 - 1 && row < g.ring_r1 + 1 && col >= g.ring_c0 - 1 &&
                          col < g.ring_c1 + 1;
      wl = in_blk;
      br = in_ext && !in_blk && mg_u(g, e, ep, MG_RING, c) < g.ring_density &&
           !mg_bit(g.clear_ring, c);
    }
    v.wall[c] = wl;
    v.brick[c] = br;
    v.crate[c] = (kind == 1 && g.open_cross) ? (uint8_t)mg_bit(g.cross, c) : 0;
    v.recycle[c] = 0;
    v.owner[c] = -1;
    v.fuse[c] = 0;
    v.blast[c] = 0;
    dng[c] = 0.f;
  }
  __syncwarp();
  // ---- open obstacles (sim/mapgen.py:65-95): the n cells with the smallest
  //      keys (ties: lower cell), then the spawn neighbourhoods cleared
  if ((kind == 1 || kind == 3) && !pure && g.obst_max > 0) {
    const int n_obst =
        (int)(((uint64_t)mg_u24(g, e, ep, MG_OBST_N, 0) * (uint64_t)(g.obst_max + 1)) >> 24);
    for (int r = 0; r < n_obst; ++r) {
      uint32_t best = 0xFFFFFFFFu;
      int bc = 0x7fffffff;
      for (int c = lane; c < C; c += 32) {
        if (v.owner[c] == -2) continue;        // taken in an earlier round
        const uint32_t k = mg_u24(g, e, ep, MG_OBST_KEY, c);
        if (k < best) {
          best = k;
          bc = c;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const uint32_t ob = __shfl_xor_sync(QQT_FULL, best, o);
        const int oc = __shfl_xor_sync(QQT_FULL, bc, o);
        if (ob < best || (ob == best && oc < bc)) {
          best = ob;
          bc = oc;
        }
      }
      if (lane == 0 && bc < C) v.owner[bc] = -2;
      __syncwarp();
    }
    for (int c = lane; c < C; c += 32)
      if (v.owner[c] == -2) {
        v.owner[c] = -1;
        v.wall[c] = !mg_bit(g.clear_spawn, c);
      }
    __syncwarp();
  }
  // ---- write the planes
  for (int c = lane; c < C; c += 32) {
    const size_t gi = (size_t)e * C + c;
    st.wall[gi] = v.wall[c];
    st.brick[gi] = v.brick[c];
    st.crate[gi] = v.crate[c];
    st.recycle[gi] = 0;
    st.owner[gi] = -1;
    st.fuse[gi] = 0;
    st.bomb_blast[gi] = 0;
  }
  // ---- players (sim/torch_sim.py:200-242, 326-383, 386-420)
  const bool swap = hash_uniform(g.seed ^ ((uint64_t)e << 32) ^ (uint64_t)ep) < 0.5f;
  const bool hz = g.hazard_fraction > 0.f && mg_u(g, e, ep, MG_HAZARD, 0) < g.hazard_fraction;
  const int si = kind == 0 ? 0 : (kind == 2 ? 2 : (kind == 1 ? 1 : 0));
  const int ak = kind == 1 ? 1 : (kind == 3 ? 2 : 0);
  float py = 0.f, px = 0.f;
  int64_t bcap_out = 0;
  if (lane < P) {
    const int p = lane;
    const size_t i = (size_t)p * N + e;
    const int src = (swap && p < 2) ? 1 - p : p;
    py = g.spawn[si][src][0];
    px = g.spawn[si][src][1];
    st.pos[((size_t)p * 2) * N + e] = py;
    st.pos[((size_t)p * 2 + 1) * N + e] = px;
    int64_t bb = st.bombs_cap[i];
    if (p < 2) {
      int64_t zz;
      float ss;
      bb = g.start_bombs[ak];
      zz = g.start_blast[ak];
      ss = g.start_spd[ak];
      if (p == 1) {
        const int64_t bo = g.opp_boost ? g.opp_boost[e] : 0;
        if (bo == 2) {
          bb = g.opp_bombs2;
          zz = g.opp_blast2;
          ss = g.opp_spd2;
        } else if (bo == 1) {
          bb = (int64_t)fminf(rintf(__fmul_rn((float)bb, g.opp_mult)), (float)g.bombs_max);
          zz = (int64_t)fminf(rintf(__fmul_rn((float)zz, g.opp_mult)), (float)g.blast_max);
          ss = fminf(__fmul_rn(ss, g.opp_mult), g.spd_max);
        }
      }
      st.blast_cap[i] = zz;
      st.spd_g[i] = ss;
      st.lo_bombs[i] = bb;
      st.lo_blast[i] = zz;
      st.lo_spd[i] = ss;
    }
    if (hz) bb = 0;                        // hazard env: no bombs for anyone
    st.bombs_cap[i] = bb;
    bcap_out = bb;
    st.alive[i] = 1;
    st.hp[i] = (uint8_t)cfg.max_hp;
    st.since_bomb[i] = cfg.place_dist_cooldown;
    st.invuln[i] = 0;
    st.pending_lost[i] = 0;
    st.combo[i] = 0;
    st.last_hit[i] = -1000000000LL;
  }
  if (lane == 0) {
    st.t[e] = 0;
    st.hazard[e] = hz ? 1 : 0;
    if (g.corridor_mode) st.crate_prob[e] = g.crate_prob_kind[kind == 1 ? 1 : (kind == 2 ? 2 : 0)];
    if (g.is_open) g.is_open[e] = (g.corridor_mode && kind == 1) ? 1 : 0;
    if (g.map_kind) g.map_kind[e] = (kind == 1 || kind == 3) ? 1 : (kind == 2 ? 2 : 0);
    g.episode[e] = ep + 1;
  }
  // ---- the new episode's observation row and legal masks
  if (OBS) {
    __syncwarp();
    observe_env<__half, false>(cfg, v, e, pinfo, dng, 0, py, px, true, 0, bcap_out, 0, ft, obs,
                               nullptr, mm, bm);
    // the rewritten row's K-tile flags: every tile (flags may over-report)
    if (obs_tiles && lane < 4) obs_tiles[(size_t)e * 4 + lane] = ~0u;
  }
}

}  // namespace qqt

using namespace qqt;

extern "C" int qqt_map_reset(const QqtCfg* cfg, const QqtState* st, const QqtMapGen* mg,
                             const uint8_t* done, void* obs, uint8_t* mm, uint8_t* bm,
                             uint32_t* obs_tiles, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if (!st || !mg || !done || !mg->episode) return QQT_E_ARG;
  if (mg->n_edge < 0 || mg->n_edge > 4 || mg->obst_max < 0) return QQT_E_ARG;
  const bool with_obs = obs != nullptr;
  if (with_obs && (!mm || !bm || cfg->obs_fp32 ||
                   cfg->obs_stride < cfg->obs_channels * cfg->height * cfg->width))
    return QQT_E_ARG;
  const int C = cfg->height * cfg->width;
  const size_t sm = QQT_NWARP * reset_warp_bytes(C);
  const int blocks = (cfg->n_envs + QQT_NWARP - 1) / QQT_NWARP;
  cudaStream_t s = (cudaStream_t)stream;
  if (with_obs) {
    cudaFuncSetAttribute(k_map_reset<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k_map_reset<true><<<blocks, QQT_NWARP * 32, sm, s>>>(*cfg, *st, *mg, done, (__half*)obs, mm,
                                                         bm, obs_tiles);
  } else {
    cudaFuncSetAttribute(k_map_reset<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k_map_reset<false><<<blocks, QQT_NWARP * 32, sm, s>>>(*cfg, *st, *mg, done, nullptr, nullptr,
                                                          nullptr, nullptr);
  }
  return launch_status();
}
