// One environment tick, fused into a single kernel (replaces
// BatchedSim.step, sim/torch_sim.py:895-1261).
//
// Block = tile of 32 envs staged in shared memory; warp = one env at a time.
// Order inside an env follows the reference exactly:
//   fuse countdown -> sequential placement -> placement bonus -> since_bomb
//   -> AABB sliding -> chain explosion (initial + fixed rounds) -> bricks to
//   crates -> damage / invulnerability -> clearing -> t, done -> rewards
//   (step, hit, placement, attribute penalty, chain bonus, crate pickup and
//   growth, danger standing, combo, terminal) -> optional device reset.
// Lanes < P own one player each; lanes stride over cells / bombs otherwise.

#include "qqt_common.cuh"

namespace qqt {

struct PlayerState {
  float y, x, spd, lo_spd;
  float rb_hit, rb_grow;   // crate pickup draws of this tick
  int alive0, hp, move, bomb, flat0, placed;
  int32_t since;
  // the int64 state counters, held as 32-bit integers for the tick (caps,
  // invulnerability ticks, lost layers and combo counts are small; last_hit
  // is a tick index or its -1e9 sentinel): exact for every value below
  // 2^31 in magnitude, and written back sign-extended
  int32_t bombs_cap, blast_cap, invuln, pending, combo, last_hit, lo_b, lo_z;
};

struct PShared {
  int flat0, alive0, bomb, placed;
  int32_t bombs_cap, blast_cap;
};

// Per-warp scratch layout (byte offsets, 16-byte aligned sections).  When
// the step writes the next observation, the row is staged at offset 0 over
// the sections that are dead by then (flames, chain lists, danger stage-A
// arrays, the placement records), so that it leaves the warp as 16-byte
// stores; the player info and the danger map it reads sit after it.
struct StepLayout {
  size_t cov, trig, list, list2, qmask, cur, bombs, ps, row, pinfo, dng, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

__host__ __device__ inline StepLayout step_layout(int cells, size_t row_bytes) {
  StepLayout L;
  L.cov = 0;
  L.trig = align16(L.cov + cells);
  L.list = align16(L.trig + cells);
  L.list2 = align16(L.list + (size_t)cells * 2);
  L.qmask = align16(L.list2 + (size_t)cells * 2);        // queued bits + a counter
  L.cur = align16(L.qmask + ((size_t)(cells + 31) / 32 + 1) * 4);
  L.bombs = align16(L.cur + (size_t)cells * 12);   // cur, front, spread
  L.ps = align16(L.bombs + (size_t)cells * 2);
  const size_t dead_end = align16(L.ps + QQT_MAX_P * sizeof(PShared));
  L.row = 0;
  L.pinfo = align16(dead_end > row_bytes ? dead_end : row_bytes);
  L.dng = align16(L.pinfo + QQT_MAX_P * sizeof(PInfo));
  L.total = align16(L.dng + (size_t)cells * 4);
  return L;
}

// Observation row bytes staged per warp (0 without the fused observation).
__host__ __device__ inline size_t step_row_bytes(const QqtCfg& cfg, bool fused_obs) {
  return fused_obs ? (size_t)cfg.obs_stride * 2 : 0;
}

__host__ __device__ inline size_t step_warp_bytes(int cells, size_t row_bytes) {
  return step_layout(cells, row_bytes).total;
}

enum { PHASE_FULL = 0, PHASE_PLACE = 1, PHASE_AFTER_PLACE = 2 };

struct StepParams {
  QqtCfg cfg;
  QqtState st;
  const int64_t* actions;
  const float* rb_hit;
  const float* rb_grow;
  int* tiers;
  QqtStepOut out;
  QqtTemplate tmpl;
  int has_tmpl;
  int phase;
  uint8_t* placed_buf;   // [P][N]
  // optional fused observation of the post-step state (the next tick's
  // input): fp16 rows [N][obs_stride], masks [N][P][5] / [N][P][2]
  __half* obs;
  uint8_t* mm;
  uint8_t* bm;
  uint32_t* obs_tiles;   // [N][4] nonzero-K-tile flags of the rows, or null
};

// Key of hazard draw family j (0: bomb count, 1: cell order, 2: blast) of
// env e at tick t (counted after the step's increment).
__device__ __forceinline__ uint64_t hazard_key(uint64_t seed, int e, int64_t t, int j) {
  return seed ^ ((uint64_t)e << 20) ^ ((uint64_t)t * 0xD1B54A32D192ED03ull) ^ ((uint64_t)j << 56);
}
__device__ __forceinline__ uint64_t hazard_seed(const QqtCfg& cfg) {
  return ((uint64_t)cfg.hazard_seed_hi << 32) | cfg.hazard_seed_lo;
}

// Hazard wave of one env (sim/torch_sim.py:1404-1466), warp-wide: after
// the tick count, before the termination test.  min(count, #free) free
// cells (no wall / brick / live bomb; a player's centre cell is free
// exactly when the player is dead, later players overriding) with the
// smallest keys get a fuse-full bomb of owner P; the r-th of them takes
// blast min + floor(u_r^x * span), x = 1 - 0.8 clamp(t / ramp).  Draws:
// hash_u24 of hazard_key(seed, env, t, family).  Returns the new length of the post-step bomb list.
__device__ __forceinline__ int hazard_wave_env(const QqtCfg& cfg, const Env& v,
                                               const DangerScratch& ds, int e, int t1, int flat1,
                                               int alive, int nb_post) {
  const int lane = lane_id(), P = cfg.n_players, C = v.cells;
  // cell keys in the stage-A weight array (not used until the danger stage
  // A that follows); 0xffffffff = not free / taken
  uint32_t* hkey = reinterpret_cast<uint32_t*>(ds.cur);
  int nfree = 0;
  for (int base = 0; base < C; base += 32) {
    const int c = base + lane;
    bool fr = c < C && !v.wall[c] && !v.brick[c] && v.fuse[c] <= 0;
    for (int q = 0; q < P; ++q) {
      const int fq = __shfl_sync(QQT_FULL, flat1, q);
      const int aq = __shfl_sync(QQT_FULL, alive, q);
      if (c < C && fq == c) fr = aq == 0;
    }
    if (c < C) hkey[c] = fr ? hash_u24(hazard_key(hazard_seed(cfg), e, t1, 1) + (uint64_t)c) : 0xFFFFFFFFu;
    nfree += __popc(__ballot_sync(QQT_FULL, fr));
  }
  __syncwarp();
  const int span = cfg.hazard_bombs_max - cfg.hazard_bombs_min + 1;
  const int cnt = cfg.hazard_bombs_min +
                  (int)(((uint64_t)hash_u24(hazard_key(hazard_seed(cfg), e, t1, 0)) * (uint64_t)span) >> 24);
  const int n_place = min(cnt, nfree);
  for (int r = 0; r < n_place; ++r) {
    uint32_t best = 0xFFFFFFFFu;
    int bc = 0x7fffffff;
    for (int c = lane; c < C; c += 32)
      if (hkey[c] < best) {
        best = hkey[c];
        bc = c;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {   // warp argmin, ties -> lower cell
      const uint32_t ob = __shfl_xor_sync(QQT_FULL, best, o);
      const int oc = __shfl_xor_sync(QQT_FULL, bc, o);
      if (ob < best || (ob == best && oc < bc)) {
        best = ob;
        bc = oc;
      }
    }
    // a dead player's cell can hold a live bomb (already in the list): it
    // is overwritten but listed once
    const bool listed = v.fuse[bc] > 0;
    __syncwarp();
    if (lane == 0) {
      const float frac = fminf(fmaxf(__fdiv_rn((float)t1, cfg.hazard_ramp_ticks), 0.f), 1.f);
      const float ex = __fsub_rn(1.f, __fmul_rn(0.8f, frac));
      const float u = (float)hash_u24(hazard_key(hazard_seed(cfg), e, t1, 2) + (uint64_t)r) *
                      (1.f / 16777216.f);
      const float vv = (float)pow((double)u, (double)ex);
      const float bspan = (float)(cfg.hazard_blast_max - cfg.hazard_blast_min + 1);
      float bl = __fadd_rn((float)cfg.hazard_blast_min, floorf(__fmul_rn(vv, bspan)));
      bl = fminf(fmaxf(bl, (float)cfg.hazard_blast_min), (float)cfg.hazard_blast_max);
      v.fuse[bc] = (int16_t)cfg.fuse;
      v.owner[bc] = (int8_t)P;
      v.blast[bc] = (int16_t)bl;
      hkey[bc] = 0xFFFFFFFFu;
      if (!listed) ds.bombs[nb_post] = (uint16_t)bc;
    }
    if (!listed) ++nb_post;
    __syncwarp();
  }
  return nb_post;
}

__device__ __forceinline__ bool placed_map_at(const PShared* ps, int P, int cell) {
  bool v = false;
  for (int i = 0; i < P; ++i)
    if (ps[i].flat0 == cell) v = ps[i].placed != 0;   // later players overwrite
  return v;
}

// PHASE, OBS (a.obs set: the fused next observation) and HZ (hazard waves
// configured) are compile-time so that each instance carries only its own
// code and registers.
// NP > 0: the player count fixed at compile time (loops over players unroll
// exactly); 0: cfg.n_players at run time.  G > 0: a G x G grid fixed at
// compile time (cell / row arithmetic by constants); 0: the config's grid.
template <int PHASE, bool OBS, bool HZ, int NP = 0, int G = 0>
__global__ void __launch_bounds__(QQT_NWARP * 32, 3) k_step(StepParams a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ FuseTables ft;
  // u8 planes (PL_WALL .. PL_RECYCLE) some env of the block changed; only
  // those are written back (fuse, owner and blast always are)
  __shared__ unsigned dirty;
  const QqtCfg& cfg = a.cfg;
  const QqtState& st = a.st;
  const int h = G > 0 ? G : cfg.height, w = G > 0 ? G : cfg.width, C = h * w, N = cfg.n_envs;
  const int P = NP > 0 ? NP : cfg.n_players;
  const int e0 = blockIdx.x * QQT_TILE_E;
  const int lane = lane_id();
  QQT_PH_START(ph_t0);
  Tile tile = carve_tile(smem, C);
  if (threadIdx.x == 0) dirty = 0;
  // the warp's env (one per warp): its per-player state and draws are loaded
  // before the tile so that their latency overlaps the staging
  static_assert(QQT_TILE_E == QQT_NWARP, "one env per warp");
  PlayerState me;
  float env_crate_prob = 0.f;
  bool env_hazard = false;
  bool env_hz = false;              // hazard-wave env (sim/torch_sim.py:1428)
  int64_t act_mv = 0, act_bo = 0;
  {
    const int e = e0 + warp_id();
    const int p = lane;
    if (e < N) {
      if (p < P) {
        const size_t i = (size_t)p * N + e;
        me.y = st.pos[((size_t)p * 2) * N + e];
        me.x = st.pos[((size_t)p * 2 + 1) * N + e];
        me.spd = st.spd_g[i];
        me.lo_spd = st.lo_spd[i];
        me.alive0 = st.alive[i];
        me.hp = st.hp[i];
        me.since = st.since_bomb[i];
        me.bombs_cap = (int32_t)st.bombs_cap[i];
        me.blast_cap = (int32_t)st.blast_cap[i];
        me.invuln = (int32_t)st.invuln[i];
        me.pending = (int32_t)st.pending_lost[i];
        me.combo = (int32_t)st.combo[i];
        me.last_hit = (int32_t)st.last_hit[i];
        me.lo_b = (int32_t)st.lo_bombs[i];
        me.lo_z = (int32_t)st.lo_blast[i];
        // the rewards' per-tick draws, loaded with the rest of the player state
        me.rb_hit = cfg.corridor ? a.rb_hit[(size_t)e * P + p] : 0.f;
        me.rb_grow = cfg.corridor ? a.rb_grow[(size_t)e * P + p] : 0.f;
      }
      env_crate_prob = cfg.corridor ? st.crate_prob[e] : 0.f;
      env_hazard = cfg.crate_speed_only && st.hazard[e];
      env_hz = HZ && st.hazard[e];
    }
  }
  // the fused observation's fuse tables (warp 0 writes them) are visible
  // to every warp after the barrier below
  if (OBS) fuse_tables(ft, a.cfg.fuse_f, a.cfg.obs_growth_bombs_max);
  load_tile(tile, st, N, e0, PL_ALL);
  __syncthreads();
  QQT_PH_AT(2, 0, ph_t0, (blockIdx.x & 3) == 0 && lane == 0);
  QQT_PH(2, 16, (blockIdx.x & 3) == 0 && lane == 0);
  // Launched as a programmatic dependent (launch_step): the state staged
  // above is no kernel's output but the previous step's, so it may be read
  // while the kernel before this one (the policy, which triggers its
  // dependents once its first layer is done) still runs.  The actions it
  // writes are read only after this wait, and nothing is written before it.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  {
    const int e = e0 + warp_id();
    if (e < N && lane < P) {
      act_mv = a.actions[((size_t)e * P + lane) * 2];
      act_bo = a.actions[((size_t)e * P + lane) * 2 + 1];
    }
  }
  const StepLayout L = step_layout(C, step_row_bytes(cfg, OBS));
  uint8_t* wb = smem + tile_bytes(C) + (size_t)warp_id() * L.total;
  uint8_t* cov = wb + L.cov;
  uint8_t* trig = wb + L.trig;
  uint16_t* list = (uint16_t*)(wb + L.list);
  uint16_t* list2 = (uint16_t*)(wb + L.list2);
  uint32_t* qmask = (uint32_t*)(wb + L.qmask);            // bomb queued for the next round
  int* qcount = (int*)(qmask + (C + 31) / 32);
  DangerScratch ds;
  ds.cur = (float*)(wb + L.cur);
  ds.front = ds.cur + C;
  ds.spread = ds.front + C;
  ds.bombs = (uint16_t*)(wb + L.bombs);
  PShared* ps = (PShared*)(wb + L.ps);
  PInfo* pinfo = (PInfo*)(wb + L.pinfo);
  float* dng = (float*)(wb + L.dng);
  const int tiers = PHASE == PHASE_PLACE ? 0 : *a.tiers;
  const float INF = __int_as_float(0x7f800000);

  for (int s = warp_id(); s < QQT_TILE_E; s += QQT_NWARP) {
    const int e = e0 + s;
    if (e >= N) break;
    const Env v = env_view(tile, s, h, w);
    const int p = lane;
    if (p < P) {
      me.alive0 = me.alive0 != 0;
      me.move = (int)max(min(act_mv, (int64_t)1 << 20), -((int64_t)1 << 20));
      me.bomb = act_bo == 1 ? 1 : 0;
      me.flat0 = center_cell(me.y, me.x, h, w);
      me.placed = 0;
    }
    QQT_PH(2, 1, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 1-2. countdown and sequential placement
    int ns0 = -1;                     // explosion sources in `list` (-1: not yet)
    if (PHASE != PHASE_AFTER_PLACE) {
      // one pass: countdown, live bombs per owner, this tick's explosion
      // sources (fuse reached 0, owner set) compacted into `list`
      // live bombs per owner: one ballot per player and 32 cells
      int live[QQT_MAX_P] = {0, 0, 0, 0};
      ns0 = 0;
#pragma unroll
      for (int base = 0; base < C; base += 32) {
        const int c = base + lane;
        bool src = false;
        int f = 0, o = -1;
        if (c < C) {
          f = v.fuse[c];
          if (f > 0) v.fuse[c] = (int16_t)(--f);
          o = v.owner[c];
          src = f == 0 && o >= 0;
          cov[c] = 0;
          trig[c] = src ? 1 : 0;
        }
#pragma unroll
        for (int q = 0; q < QQT_MAX_P; ++q)
          if (q < P) live[q] += __popc(__ballot_sync(QQT_FULL, f > 0 && o == q));
        const unsigned m = __ballot_sync(QQT_FULL, src);
        if (src) list[ns0 + __popc(m & ((1u << lane) - 1u))] = (uint16_t)c;
        ns0 += __popc(m);
      }
      if (lane < (C + 31) / 32 + 1) qmask[lane] = 0;   // queue bits and counter
      if (p < P) {
        ps[p].flat0 = me.flat0;
        ps[p].alive0 = me.alive0;
        ps[p].bomb = me.bomb;
        ps[p].bombs_cap = me.bombs_cap;
        ps[p].blast_cap = me.blast_cap;
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int q = 0; q < QQT_MAX_P; ++q) {
          if (q >= P) break;
          const int idx = ps[q].flat0;
          const bool ok = ps[q].alive0 && ps[q].bomb && v.fuse[idx] <= 0 && !v.brick[idx] &&
                          live[q] < ps[q].bombs_cap;
          ps[q].placed = ok;
          if (ok) {
            v.fuse[idx] = (int16_t)cfg.fuse;
            v.owner[idx] = (int8_t)q;
            v.blast[idx] = (int16_t)ps[q].blast_cap;
            if (trig[idx]) {          // it replaced a bomb exploding now: no source
              trig[idx] = 0;
              for (int i = 0; i < ns0; ++i)
                if (list[i] == idx) list[i] = 0xffff;
            }
          }
        }
      }
      __syncwarp();
      if (p < P) me.placed = ps[p].placed;
      if (PHASE == PHASE_PLACE) {
        if (p < P) a.placed_buf[(size_t)p * N + e] = (uint8_t)me.placed;
        int mb = cfg.blast;
        for (int c = lane; c < C; c += 32) mb = max(mb, (int)v.blast[c]);
        mb = warp_max(mb);
        if (lane == 0) atomicMax(a.tiers, mb);
        continue;
      }
    } else {
      ns0 = -1;                       // sources are compacted below
      if (p < P) {
        me.placed = a.placed_buf[(size_t)p * N + e];
        ps[p].flat0 = me.flat0;
        ps[p].alive0 = me.alive0;
        ps[p].bomb = me.bomb;
        ps[p].bombs_cap = me.bombs_cap;
        ps[p].blast_cap = me.blast_cap;
        ps[p].placed = me.placed;
      }
      __syncwarp();
    }
    const float a0f = (p < P && me.alive0) ? 1.f : 0.f;

    QQT_PH(2, 2, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 3. placement bonus (sim/torch_sim.py:1263-1355)
    float bonus = 0.f;
    if (p < P) {
      float cover = 0.f, chain = 0.f, dist = 0.f;
      if (me.placed) {
        const int s0 = me.flat0;
        const int b = blast_of(v, s0, cfg.blast);
        const int r0 = s0 / w, c0 = s0 - r0 * w;
        for (int d = -1; d < 4; ++d) {
          int r = r0, cc = c0;
          for (int k = (d < 0 ? 0 : 1); k <= (d < 0 ? 0 : b); ++k) {
            if (d >= 0) {
              r += dir_dr(d);
              cc += dir_dc(d);
              if (r < 0 || r >= h || cc < 0 || cc >= w) break;
            }
            const int q = r * w + cc;
            if (d >= 0 && v.wall[q]) break;
            for (int o = 0; o < P; ++o)
              if (o != p && ps[o].flat0 == q && ps[o].alive0) cover = __fadd_rn(cover, 1.f);
            const int fq = v.fuse[q];
            if (fq > 0 && v.owner[q] >= 0 && !placed_map_at(ps, P, q)) {
              // fq / fuse from the fuse table when it was built (same division)
              const float fdiv = (OBS && fq < 32) ? ft.norm[fq] : __fdiv_rn((float)fq, cfg.fuse_f);
              const float frac = fminf(fmaxf(fdiv, 0.f), 1.f);
              chain = __fadd_rn(chain, __fadd_rn(cfg.chain_time_factor,
                                                 __fmul_rn(cfg.chain_time_rest, __fsub_rn(1.f, frac))));
            }
            if (d >= 0 && (fq > 0 || v.brick[q])) break;
          }
        }
        if (cfg.place_dist_reward != 0.f && me.since >= cfg.place_dist_cooldown) {
          const float ry = (float)(s0 / w), rx = (float)(s0 % w);
          for (int o = 0; o < P; ++o) {
            if (o == p || !ps[o].alive0) continue;
            const int fo = ps[o].flat0;
            // opponent under the predicted flame earns cover, not distance
            bool under = fo == s0;
            const int orow = fo / w, ocol = fo % w;
            if (!under && (orow == r0 || ocol == c0)) {
              const int d = orow == r0 ? (ocol > c0 ? 3 : 2) : (orow > r0 ? 1 : 0);
              const int dist_cells = abs(orow - r0) + abs(ocol - c0);
              int r = r0, cc = c0;
              for (int k = 1; k <= b && k <= dist_cells; ++k) {
                r += dir_dr(d);
                cc += dir_dc(d);
                const int q = r * w + cc;
                if (v.wall[q]) break;
                if (k == dist_cells) under = true;
                if (v.fuse[q] > 0 || v.brick[q]) break;
              }
            }
            const float dy = __fsub_rn(ry, (float)orow), dx = __fsub_rn(rx, (float)ocol);
            const float dd = sqrtf(__fadd_rn(__fmul_rn(dy, dy), __fmul_rn(dx, dx)));
            if (!under && dd < cfg.place_dist_radius) {
              const float gain = fmaxf(__fsub_rn(1.f, __fdiv_rn(dd, cfg.place_dist_radius)), 0.f);
              dist = __fadd_rn(dist, gain);
            }
          }
        }
      }
      bonus = __fmul_rn(__fadd_rn(__fadd_rn(__fmul_rn(cfg.place_cover_reward, cover),
                                            __fmul_rn(cfg.place_dist_reward, dist)),
                                  __fmul_rn(cfg.place_chain_reward, chain)),
                        a0f);
      // ---- 4. passivity counter
      me.since = me.placed ? 0 : me.since + 1;
    }
    QQT_PH(2, 3, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 5. movement (sim/move.py:234-279).  Both axes slide from the old
    //      position, so lane p resolves player p along the rows and lane
    //      P + p along the columns at the same time.
    {
      const int pl = lane < P ? lane : (lane < 2 * P ? lane - P : 0);
      const float y0 = __shfl_sync(QQT_FULL, me.y, pl), x0 = __shfl_sync(QQT_FULL, me.x, pl);
      const float spd = __shfl_sync(QQT_FULL, me.spd, pl);
      const int move = __shfl_sync(QQT_FULL, me.move, pl);
      const int alive0 = __shfl_sync(QQT_FULL, me.alive0, pl);
      const int mv = min(max(move, 0), 4);
      float ty = 0.f, tx = 0.f;
      if (mv == 0) ty = -cfg.step_len;
      if (mv == 1) ty = cfg.step_len;
      if (mv == 2) tx = -cfg.step_len;
      if (mv == 3) tx = cfg.step_len;
      const bool moving = alive0 && move != 4;
      const float dy = moving ? __fmul_rn(ty, spd) : 0.f;
      const float dx = moving ? __fmul_rn(tx, spd) : 0.f;
      float res = 0.f;
      if (lane < 2 * P) {
        const bool vert = lane < P;
        const float d = vert ? dy : dx;
        res = resolve_axis(v, __fadd_rn(vert ? y0 : x0, d), d, vert ? x0 : y0, y0, x0, cfg.radius,
                           vert);
      }
      const float nx = __shfl_sync(QQT_FULL, res, (lane + P) & 31);
      if (p < P) {
        const float oy = dy != 0.f ? res : me.y;
        const float ox = dx != 0.f ? nx : me.x;
        me.y = fminf(fmaxf(oy, cfg.radius), cfg.h_minus_rad);
        me.x = fminf(fmaxf(ox, cfg.radius), cfg.w_minus_rad);
      }
    }

    QQT_PH(2, 4, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 6. chain explosion (sim/blast.py:101-155).  Round r triggers the
    //      live bombs covered by the flames so far; a flame that covers a
    //      live untriggered bomb queues it (once) for the next round, so a
    //      round reads the queue instead of scanning the board.
    {
      int ns = ns0;
      if (ns < 0) {
        for (int c = lane; c < C; c += 32) {
          cov[c] = 0;
          trig[c] = (v.fuse[c] == 0 && v.owner[c] >= 0) ? 1 : 0;
        }
        if (lane < (C + 31) / 32 + 1) qmask[lane] = 0;
        __syncwarp();
        ns = warp_compact(C, list, [&](int c) { return trig[c] != 0; });
      }
      __syncwarp();
      uint16_t* cur_list = list;
      uint16_t* next_list = list2;
      for (int r = 0; r <= cfg.resolve_rounds; ++r) {
        // round 0 emits the sources; round r >= 1 triggers the queue first
        if (r > 0) {
          ns = *qcount;
          __syncwarp();
          if (ns == 0) break;
          for (int i = lane; i < ns; i += 32) trig[cur_list[i]] = 1;
          if (lane == 0) *qcount = 0;
          __syncwarp();
        }
        for (int i = lane; i < ns; i += 32) {
          const int c = cur_list[i];
          if (c == 0xffff) continue;
          emit_flame_queue(v, c, blast_of(v, c, cfg.blast), tiers, cov, trig, qmask, qcount,
                           next_list);
        }
        __syncwarp();
        uint16_t* tmp = cur_list;
        cur_list = next_list;
        next_list = tmp;
      }
    }

    // ---- 7. chain bonus (off by default) needs owners before clearing
    float chain_bonus = 0.f;
    if (cfg.chain_blast_bonus != 0.f) {
      int fired[QQT_MAX_P] = {0, 0, 0, 0}, cross[QQT_MAX_P] = {0, 0, 0, 0};
      for (int c = lane; c < C; c += 32) {
        if (!trig[c]) continue;
        const int o = v.owner[c];
        const bool nat = v.fuse[c] == 0;
        for (int q = 0; q < P; ++q) {
          if (nat && o == q) fired[q] = 1;
          if (!nat && o != q) cross[q]++;
        }
      }
      for (int q = 0; q < QQT_MAX_P; ++q) {
        const int f = warp_max(fired[q]);
        const int x = warp_sum(cross[q]);
        if (q == p) chain_bonus = __fmul_rn(cfg.chain_blast_bonus, (float)(x * f));
      }
    }

    // ---- 8. (bricks burnt: in the clearing pass below; damage reads only
    //      the flame plane)

    QQT_PH(2, 5, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 9. damage and invulnerability
    int flat1 = 0, hp_new = 0, alive = 0, died = 0, lost_hp = 0;
    if (p < P) {
      flat1 = center_cell(me.y, me.x, h, w);
      const bool hit = me.alive0 && cov[flat1];
      const bool hit_eff = hit && me.invuln <= 0;
      hp_new = max(me.hp - (hit_eff ? 1 : 0), 0);
      died = hit_eff && hp_new == 0;
      lost_hp = hp_new < me.hp;
      alive = me.alive0 && !died;
      me.invuln = me.invuln - 1 > 0 ? me.invuln - 1 : 0;
      if (hit_eff) me.invuln = cfg.invuln_ticks;
    }
    __syncwarp();
    QQT_PH(2, 6, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 8 + 10. one pass: burnt bricks become crates on corridor maps,
    //      exploded bombs are cleared, and the bombs left are compacted for
    //      the danger-standing penalty below
    int nb_post = 0;
    int post_live[QQT_MAX_P] = {0, 0, 0, 0};
#pragma unroll
    for (int base = 0; base < C; base += 32) {
      const int c = base + lane;
      bool bomb = false;
      bool burnt = false;
      int o = -1;
      if (c < C) {
        if (cov[c]) {
          burnt = v.brick[c] != 0;
          if (cfg.corridor && burnt) v.crate[c] = 1;
          v.brick[c] = 0;
        }
        if (trig[c]) {
          v.fuse[c] = 0;
          v.owner[c] = -1;
          v.blast[c] = 0;
        }
        bomb = v.fuse[c] > 0;
        o = v.owner[c];
      }
#pragma unroll
      for (int q = 0; q < QQT_MAX_P; ++q)
        if (q < P) post_live[q] += __popc(__ballot_sync(QQT_FULL, bomb && o == q));
      if (__any_sync(QQT_FULL, burnt) && lane == 0) atomicOr(&dirty, PL_BRICK | PL_CRATE);
      const unsigned m = __ballot_sync(QQT_FULL, bomb);
      if (bomb) ds.bombs[nb_post + __popc(m & ((1u << lane) - 1u))] = (uint16_t)c;
      nb_post += __popc(m);
    }
    QQT_PH(2, 7, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 11. t and done
    const int64_t t1 = st.t[e] + 1;
    // ---- hazard wave (sim/torch_sim.py:1404-1466)
    if (HZ && env_hz && t1 > 0 && t1 % cfg.hazard_wave_ticks == 0)
      nb_post = hazard_wave_env(cfg, v, ds, e, (int)t1, flat1, alive, nb_post);
    const unsigned amask = __ballot_sync(QQT_FULL, p < P && alive);
    const int n_alive = __popc(amask);
    const bool done = n_alive <= 1 || t1 >= cfg.max_steps;

    QQT_PH(2, 8, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- 12. rewards
    const float dmg = (p < P) ? (float)max(me.hp - hp_new, 0) : 0.f;
    float tot_dmg = 0.f, tot_hp = 0.f;
    for (int q = 0; q < P; ++q) {
      tot_dmg = __fadd_rn(tot_dmg, __shfl_sync(QQT_FULL, dmg, q));
      tot_hp = __fadd_rn(tot_hp, __shfl_sync(QQT_FULL, (float)hp_new, q));
    }
    const float dealt = __fsub_rn(tot_dmg, dmg);
    const float coef = cfg.explore_coef;
    float reward = 0.f;
    int stood = 0;
    if (p < P) {
      reward = __fadd_rn(__fsub_rn(__fadd_rn(__fmul_rn(-cfg.step_penalty, a0f),
                                             __fmul_rn(cfg.hit_reward, dealt)),
                                   __fmul_rn(cfg.hit_reward, dmg)),
                         __fmul_rn(__fmul_rn(coef, bonus), a0f));
      if (cfg.hit_attr_penalty > 0) {
        const bool hit_any = dmg > 0.f && me.alive0;
        const int32_t pen = cfg.hit_attr_penalty;
        const int32_t nb = max(me.bombs_cap - pen, me.lo_b);
        const int32_t nz = max(me.blast_cap - pen, me.lo_z);
        const float nsp = fmaxf(__fsub_rn(me.spd, cfg.pen_speed), me.lo_spd);
        const float lostf = __fadd_rn((float)((me.bombs_cap - nb) + (me.blast_cap - nz)),
                                      rintf(__fdiv_rn(__fsub_rn(me.spd, nsp), cfg.growth_speed_step)));
        if (hit_any) {
          me.bombs_cap = nb;
          me.blast_cap = nz;
          me.spd = nsp;
          me.pending += (int32_t)lostf;
        }
      }
      reward = __fadd_rn(reward, __fmul_rn(__fmul_rn(coef, chain_bonus), a0f));
      if (cfg.corridor) {
        stood = v.crate[flat1] != 0;
        reward = __fadd_rn(reward, __fmul_rn(__fmul_rn(cfg.brick_reward, stood ? 1.f : 0.f), a0f));
        const bool rec = v.recycle[flat1] != 0;
        const float prob = rec ? cfg.recycle_crate_prob : env_crate_prob;
        const bool hits = stood && me.rb_hit < prob && me.alive0;
        int attr = (int)floorf(__fmul_rn(me.rb_grow, 3.f));
        if (env_hazard) attr = 2;
        const int32_t add_b = (hits && attr == 0) ? 1 : 0;
        const int32_t add_z = (hits && attr == 1) ? 1 : 0;
        const float add_s = (hits && attr == 2) ? 1.f : 0.f;
        me.bombs_cap = min(me.bombs_cap + add_b, cfg.growth_bombs_max);
        me.blast_cap = min(me.blast_cap + add_z, cfg.growth_blast_max);
        me.spd = fminf(__fadd_rn(me.spd, __fmul_rn(add_s, cfg.growth_speed_step)), cfg.growth_speed_max);
      }
    }
    __syncwarp();
    if (cfg.corridor && p < P && (v.crate[flat1] || v.recycle[flat1])) {
      v.crate[flat1] = 0;
      v.recycle[flat1] = 0;
      atomicOr(&dirty, PL_CRATE | PL_RECYCLE);
    }
    __syncwarp();
    QQT_PH(2, 9, (blockIdx.x & 3) == 0 && lane == 0);
    // danger standing penalty on the post-step state (sim/torch_sim.py:1163-1182)
    {
      int max_b = 0;
      danger_stage_a(v, ds, cfg.fuse_f, cfg.blast, cfg.danger_rounds, &max_b, nb_post,
                     OBS ? ft.weight : nullptr);
      const float standing = danger_at_players(v, ds, flat1, cfg.blast, max_b, P);
      if (p < P)
        reward = __fsub_rn(reward, __fmul_rn(__fmul_rn(cfg.danger_penalty, standing), a0f));
    }
    QQT_PH(2, 10, (blockIdx.x & 3) == 0 && lane == 0);
    const bool death_done = done && n_alive == 1;
    const bool all_alive = done && n_alive == P;
    int winner = 0;
    if (p < P) {
      if (cfg.combo_on) {
        const int32_t c = me.combo;
        int64_t gap = t1 - me.last_hit;
        if (gap < 0) gap = 0;
        const float factor = powf(cfg.combo_gap_factor, (float)gap);
        const int32_t inc = dealt > 0.f ? 1 : 0;
        const int32_t now = (c + inc) * inc;
        const float pts = __fmul_rn(__fmul_rn(__fmul_rn((float)now, cfg.combo_reward), factor),
                                    fminf(dealt, 1.f));
        reward = __fadd_rn(reward, __fmul_rn(pts, a0f));
        if (inc) {
          me.combo = now;
          me.last_hit = (int32_t)t1;
        }
        if (dmg > 0.f) me.combo = 0;
      }
      winner = death_done && alive && n_alive == 1;
      const int loser = death_done && !alive && n_alive == 1;
      const float hpf = (float)hp_new;
      // (x / 1 is x exactly: no division for two players)
      const float others = __fsub_rn(tot_hp, hpf);
      const float diff = __fsub_rn(hpf, P == 2 ? others : __fdiv_rn(others, (float)(P - 1)));
      const float aa = all_alive ? 1.f : 0.f;
      if (!cfg.win_hp_scaled) {
        reward = __fadd_rn(reward, __fmul_rn(cfg.win_bonus,
                                             __fsub_rn(winner ? 1.f : 0.f, loser ? 1.f : 0.f)));
        if (cfg.timeout_draw)
          reward = __fadd_rn(reward, __fmul_rn(__fmul_rn(__fmul_rn(cfg.win_bonus_per_hp, diff), aa), coef));
      } else {
        const float base = __fmul_rn(cfg.win_bonus_per_hp, diff);
        const float scale = cfg.timeout_draw ? coef : 1.f;
        reward = __fadd_rn(reward, __fadd_rn(__fmul_rn(base, death_done ? 1.f : 0.f),
                                             __fmul_rn(__fmul_rn(base, aa), scale)));
      }
    }

    QQT_PH(2, 11, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- outputs
    if (p < P) {
      const size_t ri = (size_t)e * P + p;
      if (a.out.reward) a.out.reward[ri] = reward;
      if (a.out.died) a.out.died[ri] = (uint8_t)died;
      if (a.out.hit) a.out.hit[ri] = (uint8_t)(lost_hp && !done);
      if (a.out.winner) a.out.winner[ri] = (uint8_t)winner;
    }
    if (lane == 0) {
      if (a.out.done) a.out.done[e] = done;
      if (a.out.n_alive) a.out.n_alive[e] = n_alive;
      if (a.out.reset_mask) a.out.reset_mask[e] = (done && a.has_tmpl) ? 1 : 0;
    }
    if (a.out.covered || a.out.triggered) {
      for (int c = lane; c < C; c += 32) {
        if (a.out.covered) a.out.covered[(size_t)e * C + c] = cov[c];
        if (a.out.triggered) a.out.triggered[(size_t)e * C + c] = trig[c];
      }
    }

    QQT_PH(2, 12, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- device reset to the env's template (no host round trip)
    int64_t t_out = t1;
    if (done && a.has_tmpl) {
      const QqtTemplate& tp = a.tmpl;
      if (lane == 0) atomicOr(&dirty, PL_ALL);
      for (int c = lane; c < C; c += 32) {
        const size_t g = (size_t)e * C + c;
        v.wall[c] = tp.wall[g];
        v.brick[c] = tp.brick[g];
        v.crate[c] = tp.crate ? tp.crate[g] : 0;
        v.recycle[c] = 0;
        v.fuse[c] = 0;
        v.owner[c] = -1;
        v.blast[c] = 0;
      }
      const int64_t epi = tp.episode[e];
      const bool swap = tp.swap_spawns &&
                        hash_uniform(tp.seed ^ ((uint64_t)e << 32) ^ (uint64_t)epi) < 0.5f;
      if (p < P) {
        const int src = (swap && p < 2) ? 1 - p : p;
        const size_t i = (size_t)p * N + e;
        me.y = tp.spawn[((size_t)src * 2) * N + e];
        me.x = tp.spawn[((size_t)src * 2 + 1) * N + e];
        alive = 1;
        hp_new = cfg.max_hp;
        me.since = tp.since_bomb0;
        me.invuln = 0;
        me.pending = 0;
        me.combo = 0;
        me.last_hit = -1000000000;
        me.bombs_cap = (int32_t)tp.bombs_cap[i];
        me.blast_cap = (int32_t)tp.blast_cap[i];
        me.spd = tp.spd[i];
        me.lo_b = me.bombs_cap;
        me.lo_z = me.blast_cap;
        me.lo_spd = me.spd;
      }
      if (lane == 0) {
        tp.episode[e] = epi + 1;
        st.crate_prob[e] = tp.crate_prob[e];
        st.hazard[e] = 0;
      }
      t_out = 0;
    }
    QQT_PH(2, 13, (blockIdx.x & 3) == 0 && lane == 0);
    // ---- fused observation of the post-step (or reset) state: the next
    //      tick's observation row and legal masks (sim/obs.py:25-229).  The
    //      danger map reuses the danger-standing stage A (same planes); an
    //      env reset to its template has no bombs.
    if (OBS) {
      const bool reset = done && a.has_tmpl;
      danger_paint(v, ds, reset ? 0 : nb_post, cfg.blast, dng);
      int my_live = 0;    // live bombs of this lane's player (lanes < P)
#pragma unroll
      for (int q = 0; q < QQT_MAX_P; ++q)
        if (lane == q && !reset) my_live = post_live[q];
      observe_env<__half, true, NP, G>(cfg, v, e, pinfo, dng, my_live, me.y, me.x, alive != 0, me.invuln,
                          me.bombs_cap, t_out, ft, a.obs, nullptr, a.mm, a.bm,
                          (__half*)(wb + L.row), a.obs_tiles);
    }
    QQT_PH(2, 14, (blockIdx.x & 3) == 0 && lane == 0);
    if (p < P) {
      const size_t i = (size_t)p * N + e;
      st.pos[((size_t)p * 2) * N + e] = me.y;
      st.pos[((size_t)p * 2 + 1) * N + e] = me.x;
      st.alive[i] = (uint8_t)alive;
      st.hp[i] = (uint8_t)hp_new;
      st.since_bomb[i] = me.since;
      st.bombs_cap[i] = me.bombs_cap;
      st.blast_cap[i] = me.blast_cap;
      st.spd_g[i] = me.spd;
      st.invuln[i] = me.invuln;
      st.pending_lost[i] = me.pending;
      st.combo[i] = me.combo;
      st.last_hit[i] = me.last_hit;
      if (done && a.has_tmpl) {
        st.lo_bombs[i] = me.lo_b;
        st.lo_blast[i] = me.lo_z;
        st.lo_spd[i] = me.lo_spd;
      }
    }
    QQT_PH(2, 15, (blockIdx.x & 3) == 0 && lane == 0);
    if (lane == 0) st.t[e] = t_out;
    __syncwarp();
  }
  __syncthreads();
  const unsigned planes = (PL_FUSE | PL_OWNER | PL_BLAST) |
                          (PHASE == PHASE_PLACE ? 0u : dirty);
  store_tile(tile, st, N, e0, planes);
  QQT_PH(2, 17, (blockIdx.x & 3) == 0 && lane == 0);
}

// Crate recycling on the device (sim/torch_sim.py:549-596 semantics with a
// counter-based RNG): for each player with lost layers, pick
// min(lost, available) distinct cells uniformly among free cells outside the
// exclusion set -- every free cell draws a random key and the k smallest
// keys win -- mark them crate + recycled, clear the pending count.
// One warp per env, lanes over cells.
struct ExclBits {
  uint32_t w[(QQT_MAX_CELLS + 31) / 32];
};

__global__ void k_flush_recycle(QqtCfg cfg, QqtState st, ExclBits ex, uint64_t seed,
                                uint64_t counter) {
  const int e = blockIdx.x * (blockDim.x >> 5) + warp_id();
  const int N = cfg.n_envs, P = cfg.n_players, C = cfg.height * cfg.width;
  const int lane = lane_id();
  if (e >= N) return;
  for (int p = 0; p < P; ++p) {
    const int64_t lost = st.pending_lost[(size_t)p * N + e];
    if (lost <= 0) continue;
    const uint64_t key = seed ^ (counter * 0x9E3779B97F4A7C15ull) ^ ((uint64_t)e << 20) ^
                         ((uint64_t)p << 52) ^ ((uint64_t)st.t[e] * 0xD1B54A32D192ED03ull);
    // per-lane keys for its cells (up to 14 cells per lane for 21x21)
    float kv[(QQT_MAX_CELLS + 31) / 32];
    int nav = 0;
#pragma unroll
    for (int i = 0; i < (QQT_MAX_CELLS + 31) / 32; ++i) {
      const int c = lane + 32 * i;
      float k = 2.f;                                    // 2 = not available
      if (c < C) {
        const size_t g = (size_t)e * C + c;
        if (!st.wall[g] && !st.brick[g] && !((ex.w[c >> 5] >> (c & 31)) & 1u)) {
          k = hash_uniform(key + (uint64_t)c);
          ++nav;
        }
      }
      kv[i] = k;
    }
    nav = warp_sum(nav);
    const int need = (int)min((int64_t)nav, lost);
    for (int r = 0; r < need; ++r) {
      float best = 2.f;
      int bc = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < (QQT_MAX_CELLS + 31) / 32; ++i)
        if (kv[i] < best) {
          best = kv[i];
          bc = lane + 32 * i;
        }
      // warp argmin (ties -> lower cell)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(QQT_FULL, best, o);
        const int oc = __shfl_xor_sync(QQT_FULL, bc, o);
        if (ob < best || (ob == best && oc < bc)) {
          best = ob;
          bc = oc;
        }
      }
      if ((bc & 31) == lane) {
        const size_t g = (size_t)e * C + bc;
        st.crate[g] = 1;
        st.recycle[g] = 1;
#pragma unroll
        for (int i = 0; i < (QQT_MAX_CELLS + 31) / 32; ++i)
          if (lane + 32 * i == bc) kv[i] = 2.f;
      }
      __syncwarp();
    }
    if (lane == 0) st.pending_lost[(size_t)p * N + e] = 0;
  }
}

}  // namespace qqt

using namespace qqt;

extern "C" int qqt_flush_recycle(const QqtCfg* cfg, const QqtState* st, const uint32_t* excl_bits,
                                 uint64_t seed, uint64_t counter, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if (!st || !excl_bits) return QQT_E_ARG;
  ExclBits ex;
  const int C = cfg->height * cfg->width;
  memset(&ex, 0, sizeof(ex));
  for (int i = 0; i < (C + 31) / 32; ++i) ex.w[i] = excl_bits[i];
  const int N = cfg->n_envs;
  k_flush_recycle<<<(N + 7) / 8, 256, 0, (cudaStream_t)stream>>>(*cfg, *st, ex, seed, counter);
  return launch_status();
}

extern "C" uint64_t qqt_step_scratch_bytes(const QqtCfg* cfg) {
  if (!cfg) return 0;
  return ((uint64_t)cfg->n_players * cfg->n_envs + 255) / 256 * 256;
}

// QQT_STEP_PDL=0 launches the step without programmatic stream
// serialization (it then starts only once the kernel before it has ended).
static bool step_pdl_enabled() {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("QQT_STEP_PDL");
    env = (e && e[0] == '0') ? 0 : 1;
  }
  return env == 1;
}

static int launch_step(const QqtCfg* cfg, const QqtState* st, const int64_t* actions,
                       const float* rb_hit, const float* rb_grow, int32_t* tiers,
                       int32_t first_step, const QqtStepOut* out, const QqtTemplate* tmpl,
                       void* scratch, void* obs, uint8_t* mm, uint8_t* bm,
                       uint32_t* obs_tiles, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if (!st || !actions || !tiers || !scratch) return QQT_E_ARG;
  if (cfg->corridor && (!rb_hit || !rb_grow)) return QQT_E_ARG;
  if (tmpl && (!tmpl->wall || !tmpl->brick || !tmpl->spawn || !tmpl->bombs_cap ||
               !tmpl->blast_cap || !tmpl->spd || !tmpl->crate_prob || !tmpl->episode))
    return QQT_E_ARG;
  if (obs && (!mm || !bm || cfg->obs_fp32 || cfg->obs_stride < cfg->obs_channels * cfg->height *
                                                                   cfg->width))
    return QQT_E_ARG;
  StepParams p;
  p.cfg = *cfg;
  p.st = *st;
  p.actions = actions;
  p.rb_hit = rb_hit;
  p.rb_grow = rb_grow;
  p.tiers = tiers;
  if (out) {
    p.out = *out;
  } else {
    memset(&p.out, 0, sizeof(p.out));
  }
  if (tmpl) {
    p.tmpl = *tmpl;
    p.has_tmpl = 1;
  } else {
    memset(&p.tmpl, 0, sizeof(p.tmpl));
    p.has_tmpl = 0;
  }
  p.placed_buf = (uint8_t*)scratch;
  p.obs = (__half*)obs;
  p.mm = mm;
  p.bm = bm;
  p.obs_tiles = obs ? obs_tiles : nullptr;
  const int C = cfg->height * cfg->width;
  const size_t sm = tile_bytes(C) + QQT_NWARP * step_warp_bytes(C, step_row_bytes(*cfg, obs != nullptr));
  const int blocks = (cfg->n_envs + QQT_TILE_E - 1) / QQT_TILE_E;
  cudaStream_t s = (cudaStream_t)stream;
  // programmatic stream serialization: the step may start (stage its tile)
  // once the kernel before it in the stream has triggered its dependents;
  // kernels that never trigger (all but the policy) serialise as usual
  const bool pdl = step_pdl_enabled();
  auto launch = [&](auto kern, int phase) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    p.phase = phase;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks, 1, 1);
    lc.blockDim = dim3(QQT_NWARP * 32, 1, 1);
    lc.dynamicSmemBytes = sm;
    lc.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&lc, kern, p);
  };
  const bool fused = obs != nullptr;
  const bool hz = cfg->hazard_on != 0;
  // the steady-state two-player tick on the 13 x 13 board of the
  // benchmark configs has its own instance
  const bool two = cfg->n_players == 2, g13 = cfg->height == 13 && cfg->width == 13;
  if (first_step) {
    cudaMemsetAsync(tiers, 0xff, sizeof(int32_t), s);   // -1
    launch(k_step<PHASE_PLACE, false, false>, PHASE_PLACE);
    if (fused) {
      if (hz) launch(k_step<PHASE_AFTER_PLACE, true, true>, PHASE_AFTER_PLACE);
      else launch(k_step<PHASE_AFTER_PLACE, true, false>, PHASE_AFTER_PLACE);
    } else {
      if (hz) launch(k_step<PHASE_AFTER_PLACE, false, true>, PHASE_AFTER_PLACE);
      else launch(k_step<PHASE_AFTER_PLACE, false, false>, PHASE_AFTER_PLACE);
    }
  } else if (fused) {
    if (hz) launch(k_step<PHASE_FULL, true, true>, PHASE_FULL);
    else if (two && g13) launch(k_step<PHASE_FULL, true, false, 2, 13>, PHASE_FULL);
    else if (two) launch(k_step<PHASE_FULL, true, false, 2>, PHASE_FULL);
    else launch(k_step<PHASE_FULL, true, false>, PHASE_FULL);
  } else {
    if (hz) launch(k_step<PHASE_FULL, false, true>, PHASE_FULL);
    else if (two && g13) launch(k_step<PHASE_FULL, false, false, 2, 13>, PHASE_FULL);
    else if (two) launch(k_step<PHASE_FULL, false, false, 2>, PHASE_FULL);
    else launch(k_step<PHASE_FULL, false, false>, PHASE_FULL);
  }
  return launch_status();
}

extern "C" int qqt_step(const QqtCfg* cfg, const QqtState* st, const int64_t* actions,
                        const float* rb_hit, const float* rb_grow, int32_t* tiers,
                        int32_t first_step, const QqtStepOut* out, const QqtTemplate* tmpl,
                        void* scratch, qqt_stream_t stream) {
  return launch_step(cfg, st, actions, rb_hit, rb_grow, tiers, first_step, out, tmpl, scratch,
                     nullptr, nullptr, nullptr, nullptr, stream);
}

extern "C" int qqt_step_observe(const QqtCfg* cfg, const QqtState* st, const int64_t* actions,
                                const float* rb_hit, const float* rb_grow, int32_t* tiers,
                                int32_t first_step, const QqtStepOut* out, const QqtTemplate* tmpl,
                                void* scratch, void* obs, uint8_t* mm, uint8_t* bm,
                                uint32_t* obs_tiles, qqt_stream_t stream) {
  if (!obs || !mm || !bm) return QQT_E_ARG;
  if (((uintptr_t)obs & 15) || ((uintptr_t)obs_tiles & 15) || (cfg && (cfg->obs_stride % 8)))
    return QQT_E_ALIGN;
  return launch_step(cfg, st, actions, rb_hit, rb_grow, tiers, first_step, out, tmpl, scratch,
                     obs, mm, bm, obs_tiles, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free step.  Some callers cannot call cudaMalloc at all: code that
// runs inside another runtime's stream capture, an embedding that hands this
// library a fixed device budget, or a host without a device allocator hook.
// qqt_step_noalloc gives them the same step as qqt_step with its scratch (the
// per-player placement flags of the first-step pass) in a fixed static device
// array instead of a caller buffer.  The array is QQT_STEP_NOALLOC_MAX bytes
// (n_envs * n_players must fit); every GPU that loads the library holds it
// until exit.
#include <mutex>

#define QQT_STEP_NOALLOC_MAX (256 * 1024)
static __device__ __align__(256) uint8_t g_step_noalloc_scratch[QQT_STEP_NOALLOC_MAX];

// Device address of the static array, looked up once per device with that
// device current (in host code the array's name is only a host-side stand-in).
static void* step_noalloc_ptr() {
  static std::mutex mu;
  static void* addr[128] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_step_noalloc_scratch) != cudaSuccess) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

extern "C" int qqt_step_noalloc(const QqtCfg* cfg, const QqtState* st, const int64_t* actions,
                                const float* rb_hit, const float* rb_grow, int32_t* tiers,
                                int32_t first_step, const QqtStepOut* out,
                                const QqtTemplate* tmpl, qqt_stream_t stream) {
  int rc = check_cfg(cfg);
  if (rc) return rc;
  if ((uint64_t)cfg->n_envs * (uint64_t)cfg->n_players > QQT_STEP_NOALLOC_MAX) return QQT_E_LIMIT;
  void* scratch = step_noalloc_ptr();
  if (!scratch) return QQT_E_LAUNCH;
  return qqt_step(cfg, st, actions, rb_hit, rb_grow, tiers, first_step, out, tmpl, scratch, stream);
}
