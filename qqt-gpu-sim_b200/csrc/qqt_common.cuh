// Shared device code of the B200 rollout engine.
//
// Work decomposition: one thread block owns a tile of QQT_TILE_E consecutive
// envs.  Planes are env-major in global memory ([env][cell]), so the block
// stages each plane of its tile as one contiguous run (coalesced 8- and
// 16-byte accesses) into shared memory with the same [env][cell] layout,
// then each warp simulates one env with its 32 lanes spread over cells /
// bombs / players.  With per-env contiguous planes, lanes walking
// consecutive cells hit distinct banks.
//
// Float arithmetic on the parity path uses the _rn intrinsics in the exact
// operation order of the reference (the library is also built with
// -fmad=false), so positions, rewards and danger match the reference bit for
// bit.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>

#include "../../include/qqt_b200.h"

#define QQT_MAX_H 21
#define QQT_MAX_W 21
#define QQT_MAX_CELLS (QQT_MAX_H * QQT_MAX_W)
#define QQT_MAX_P 4
#define QQT_TILE_E 8
#define QQT_NWARP 8
#define QQT_FULL 0xffffffffu

namespace qqt {

__device__ unsigned int g_error = 0;   // device error word (qqt_get_error)

__device__ __forceinline__ void flag_error(unsigned bits) { atomicOr(&g_error, bits); }

// Phase stamps (build.py --phase-stamps, QQT_PHASE_STAMPS): kernels append
// (kernel id, phase, SM, block, warp, globaltimer ns) records at their phase
// boundaries to a device ring that qqt_phase_read copies out; the regular
// build compiles every stamp to nothing.  Kernel ids: 1 the MLP policy, 2
// the simulator step.
#ifdef QQT_PHASE_STAMPS
#define QQT_PH_CAP 8000000u
__device__ unsigned long long g_ph[2 * QQT_PH_CAP];
__device__ unsigned int g_ph_n;
__device__ __forceinline__ unsigned long long ph_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void ph_rec(unsigned kid, unsigned ph, unsigned long long t) {
  unsigned smid;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  const unsigned i = atomicAdd(&g_ph_n, 1u);
  if (i < QQT_PH_CAP) {
    g_ph[2 * i] = ((unsigned long long)kid << 56) | ((unsigned long long)ph << 48) |
                  ((unsigned long long)smid << 32) | ((unsigned long long)blockIdx.x << 8) |
                  (threadIdx.x >> 5);
    g_ph[2 * i + 1] = t;
  }
}
#define QQT_PH_START(var) const unsigned long long var = ph_now()
#define QQT_PH(kid, ph, cond) \
  do {                        \
    if (cond) ph_rec((kid), (ph), ph_now()); \
  } while (0)
#define QQT_PH_AT(kid, ph, t, cond) \
  do {                              \
    if (cond) ph_rec((kid), (ph), (t)); \
  } while (0)
#else
#define QQT_PH_START(var) \
  do {                    \
  } while (0)
#define QQT_PH(kid, ph, cond) \
  do {                        \
  } while (0)
#define QQT_PH_AT(kid, ph, t, cond) \
  do {                              \
  } while (0)
#endif

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(QQT_FULL, v, o);
  return v;
}
__device__ __forceinline__ int warp_max(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(QQT_FULL, v, o));
  return v;
}

// Cells c in [0, n) with pred(c), ascending, written to list; returns count.
template <class F>
__device__ __forceinline__ int warp_compact(int n, uint16_t* list, F pred) {
  const int lane = lane_id();
  int count = 0;
#pragma unroll
  for (int base = 0; base < n; base += 32) {
    const int c = base + lane;
    const bool p = c < n && pred(c);
    const unsigned m = __ballot_sync(QQT_FULL, p);
    if (p) list[count + __popc(m & ((1u << lane) - 1u))] = (uint16_t)c;
    count += __popc(m);
  }
  __syncwarp();
  return count;
}

// ------------------------------------------------------------ tile staging

// Per-env planes of one block tile, [env slot][cell].
struct Tile {
  uint8_t *wall, *brick, *crate, *recycle;
  int8_t* owner;
  int16_t *fuse, *blast;
  int cells;
};

__host__ __device__ inline size_t tile_bytes(int cells) {
  // 4 u8 planes + owner + 2 i16 planes, each E * cells, 16-byte aligned
  const size_t u8 = ((size_t)QQT_TILE_E * cells + 15) & ~(size_t)15;
  const size_t i16 = ((size_t)QQT_TILE_E * cells * 2 + 15) & ~(size_t)15;
  return 5 * u8 + 2 * i16;
}

__device__ inline Tile carve_tile(uint8_t* base, int cells) {
  Tile t;
  const size_t u8 = ((size_t)QQT_TILE_E * cells + 15) & ~(size_t)15;
  const size_t i16 = ((size_t)QQT_TILE_E * cells * 2 + 15) & ~(size_t)15;
  t.wall = base;
  t.brick = base + u8;
  t.crate = base + 2 * u8;
  t.recycle = base + 3 * u8;
  t.owner = (int8_t*)(base + 4 * u8);
  t.fuse = (int16_t*)(base + 5 * u8);
  t.blast = (int16_t*)(base + 5 * u8 + i16);
  t.cells = cells;
  return t;
}

enum : unsigned {
  PL_WALL = 1, PL_BRICK = 2, PL_CRATE = 4, PL_RECYCLE = 8,
  PL_OWNER = 16, PL_FUSE = 32, PL_BLAST = 64, PL_ALL = 127
};

static_assert(QQT_TILE_E == 8, "vectorised tile transfers move 8-byte / 16-byte chunks");

// Planes are env-major ([N][C]), so a tile (envs e0 .. e0+7) is one
// contiguous run of 8 * C elements per plane, laid out in shared memory
// exactly as in global memory ([slot][cell]).  A full tile with 16-byte
// aligned plane bases moves in 8-byte (u8 planes: 8 * C bytes = C chunks)
// and 16-byte (i16 planes: 16 * C bytes = C chunks) accesses, consecutive
// threads on consecutive chunks; a partial tile element by element.
__device__ __forceinline__ bool tile_vector_ok(const QqtState& st, int n, int e0) {
  const uintptr_t a = (uintptr_t)st.wall | (uintptr_t)st.brick | (uintptr_t)st.crate |
                      (uintptr_t)st.recycle | (uintptr_t)st.owner | (uintptr_t)st.fuse |
                      (uintptr_t)st.bomb_blast;
  return e0 + QQT_TILE_E <= n && (a & 15) == 0;
}

// Global [N][C] -> shared [slot][cell] for envs e0 .. e0+E-1 (block-wide).
// Thread j moves chunk j (and j + blockDim, ...) of every requested plane:
// its loads are issued together, then stored.
__device__ inline void load_tile(const Tile& t, const QqtState& st, int n, int e0,
                                 unsigned planes) {
  const int cells = t.cells;
  if (tile_vector_ok(st, n, e0)) {
    const size_t o = (size_t)e0 * cells;   // element offset of the tile in a plane
    for (int k = threadIdx.x; k < cells; k += blockDim.x) {
      const uint2 z2 = make_uint2(0, 0);
      const uint4 z4 = make_uint4(0, 0, 0, 0);
      const uint2 wl = (planes & PL_WALL) ? reinterpret_cast<const uint2*>(st.wall + o)[k] : z2;
      const uint2 br = (planes & PL_BRICK) ? reinterpret_cast<const uint2*>(st.brick + o)[k] : z2;
      const uint2 cr = (planes & PL_CRATE) ? reinterpret_cast<const uint2*>(st.crate + o)[k] : z2;
      const uint2 rc = (planes & PL_RECYCLE) ? reinterpret_cast<const uint2*>(st.recycle + o)[k] : z2;
      const uint2 ow = (planes & PL_OWNER) ? reinterpret_cast<const uint2*>(st.owner + o)[k] : z2;
      const uint4 fu = (planes & PL_FUSE) ? reinterpret_cast<const uint4*>(st.fuse + o)[k] : z4;
      const uint4 bl = (planes & PL_BLAST) ? reinterpret_cast<const uint4*>(st.bomb_blast + o)[k] : z4;
      if (planes & PL_WALL) reinterpret_cast<uint2*>(t.wall)[k] = wl;
      if (planes & PL_BRICK) reinterpret_cast<uint2*>(t.brick)[k] = br;
      if (planes & PL_CRATE) reinterpret_cast<uint2*>(t.crate)[k] = cr;
      if (planes & PL_RECYCLE) reinterpret_cast<uint2*>(t.recycle)[k] = rc;
      if (planes & PL_OWNER) reinterpret_cast<uint2*>(t.owner)[k] = ow;
      if (planes & PL_FUSE) reinterpret_cast<uint4*>(t.fuse)[k] = fu;
      if (planes & PL_BLAST) reinterpret_cast<uint4*>(t.blast)[k] = bl;
    }
    return;
  }
  const int total = cells * min(QQT_TILE_E, n - e0);
  const size_t g0 = (size_t)e0 * cells;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const size_t g = g0 + i;
    if (planes & PL_WALL) t.wall[i] = st.wall[g];
    if (planes & PL_BRICK) t.brick[i] = st.brick[g];
    if (planes & PL_CRATE) t.crate[i] = st.crate[g];
    if (planes & PL_RECYCLE) t.recycle[i] = st.recycle[g];
    if (planes & PL_OWNER) t.owner[i] = st.owner[g];
    if (planes & PL_FUSE) t.fuse[i] = st.fuse[g];
    if (planes & PL_BLAST) t.blast[i] = st.bomb_blast[g];
  }
}

// Shared [slot][cell] -> global [N][C] (block-wide; after a __syncthreads()).
__device__ inline void store_tile(const Tile& t, const QqtState& st, int n, int e0,
                                  unsigned planes) {
  const int cells = t.cells;
  if (tile_vector_ok(st, n, e0)) {
    const size_t o = (size_t)e0 * cells;
    for (int k = threadIdx.x; k < cells; k += blockDim.x) {
      if (planes & PL_WALL)
        reinterpret_cast<uint2*>(st.wall + o)[k] = reinterpret_cast<const uint2*>(t.wall)[k];
      if (planes & PL_BRICK)
        reinterpret_cast<uint2*>(st.brick + o)[k] = reinterpret_cast<const uint2*>(t.brick)[k];
      if (planes & PL_CRATE)
        reinterpret_cast<uint2*>(st.crate + o)[k] = reinterpret_cast<const uint2*>(t.crate)[k];
      if (planes & PL_RECYCLE)
        reinterpret_cast<uint2*>(st.recycle + o)[k] = reinterpret_cast<const uint2*>(t.recycle)[k];
      if (planes & PL_OWNER)
        reinterpret_cast<uint2*>(st.owner + o)[k] = reinterpret_cast<const uint2*>(t.owner)[k];
      if (planes & PL_FUSE)
        reinterpret_cast<uint4*>(st.fuse + o)[k] = reinterpret_cast<const uint4*>(t.fuse)[k];
      if (planes & PL_BLAST)
        reinterpret_cast<uint4*>(st.bomb_blast + o)[k] = reinterpret_cast<const uint4*>(t.blast)[k];
    }
    return;
  }
  const int total = cells * min(QQT_TILE_E, n - e0);
  const size_t g0 = (size_t)e0 * cells;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const size_t g = g0 + i;
    if (planes & PL_WALL) st.wall[g] = t.wall[i];
    if (planes & PL_BRICK) st.brick[g] = t.brick[i];
    if (planes & PL_CRATE) st.crate[g] = t.crate[i];
    if (planes & PL_RECYCLE) st.recycle[g] = t.recycle[i];
    if (planes & PL_OWNER) st.owner[g] = t.owner[i];
    if (planes & PL_FUSE) st.fuse[g] = t.fuse[i];
    if (planes & PL_BLAST) st.bomb_blast[g] = t.blast[i];
  }
}

// One env's view into the tile.
struct Env {
  uint8_t *wall, *brick, *crate, *recycle;
  int8_t* owner;
  int16_t *fuse, *blast;
  int h, w, cells;
};

__device__ inline Env env_view(const Tile& t, int slot, int h, int w) {
  const int o = slot * t.cells;
  Env v;
  v.wall = t.wall + o;
  v.brick = t.brick + o;
  v.crate = t.crate + o;
  v.recycle = t.recycle + o;
  v.owner = t.owner + o;
  v.fuse = t.fuse + o;
  v.blast = t.blast + o;
  v.h = h;
  v.w = w;
  v.cells = t.cells;
  return v;
}

__device__ __forceinline__ int blast_of(const Env& v, int c, int default_blast) {
  const int b = v.blast[c];
  return b > 0 ? b : default_blast;
}

// Direction d (0 up, 1 down, 2 left, 3 right) as row / column steps,
// computed (no table: a per-lane d would serialise constant-cache reads).
__device__ __forceinline__ int dir_dr(int d) { return d == 0 ? -1 : (d == 1 ? 1 : 0); }
__device__ __forceinline__ int dir_dc(int d) { return d == 2 ? -1 : (d == 3 ? 1 : 0); }

// ------------------------------------------------------------- fire rays

// Flame of one source: its own cell (unless wall/brick) plus, when its blast
// is within the tier bound, up to `blast` cells per direction; walls stop
// the ray uncovered, solid cells (live bombs, bricks) are covered then stop
// it (sim/blast.py:43-98).  `cov` is a byte map; concurrent writers only
// store 1.
__device__ inline void emit_flame(const Env& v, int src, int blast, int tier_cap,
                                  volatile uint8_t* cov) {
  if (v.wall[src] || v.brick[src]) return;
  cov[src] = 1;
  if (blast > tier_cap) return;
  const int r0 = src / v.w, c0 = src - r0 * v.w;
  for (int d = 0; d < 4; ++d) {
    int r = r0, c = c0;
    for (int k = 1; k <= blast; ++k) {
      r += dir_dr(d);
      c += dir_dc(d);
      if (r < 0 || r >= v.h || c < 0 || c >= v.w) break;
      const int q = r * v.w + c;
      if (v.wall[q]) break;
      cov[q] = 1;
      if (v.fuse[q] > 0 || v.brick[q]) break;
    }
  }
}

// emit_flame that also queues every live, not yet triggered bomb its flame
// covers (once: bit in qmask) into next[*qcount] for the next chain round.
__device__ inline void emit_flame_queue(const Env& v, int src, int blast, int tier_cap,
                                        volatile uint8_t* cov, const volatile uint8_t* trig,
                                        uint32_t* qmask, int* qcount, uint16_t* next) {
  if (v.wall[src] || v.brick[src]) return;
  cov[src] = 1;
  if (blast > tier_cap) return;
  const int r0 = src / v.w, c0 = src - r0 * v.w;
  for (int d = 0; d < 4; ++d) {
    int r = r0, c = c0;
    for (int k = 1; k <= blast; ++k) {
      r += dir_dr(d);
      c += dir_dc(d);
      if (r < 0 || r >= v.h || c < 0 || c >= v.w) break;
      const int q = r * v.w + c;
      if (v.wall[q]) break;
      cov[q] = 1;
      if (v.fuse[q] > 0) {
        if (!trig[q]) {
          const uint32_t bit = 1u << (q & 31);
          if (!(atomicOr(qmask + (q >> 5), bit) & bit)) next[atomicAdd(qcount, 1)] = (uint16_t)q;
        }
        break;
      }
      if (v.brick[q]) break;
    }
  }
}

// ------------------------------------------------------------- danger map

// Bomb weight clamp(1 - (f-1)/FUSE, 0)^2 in float32 (sim/blast.py:218-220).
__device__ __forceinline__ float fuse_weight(int f, float fuse_f) {
  if (f <= 0) return 0.f;
  float raw = __fsub_rn(1.f, __fdiv_rn(__fsub_rn((float)f, 1.f), fuse_f));
  raw = fmaxf(raw, 0.f);
  return __fmul_rn(raw, raw);
}

// Largest weight `val` over the bombs whose flame reaches cell c (the nearest
// bomb along each direction, within its blast, through clear cells), or 0.
// Solid = bomb (fuse > 0) or brick; walls stop silently.
__device__ inline float reach_max(const Env& v, int c, const float* val, int default_blast,
                                  int max_b) {
  const int r0 = c / v.w, c0 = c - r0 * v.w;
  float best = 0.f;
  for (int d = 0; d < 4; ++d) {
    int r = r0, cc = c0;
    for (int k = 1; k <= max_b; ++k) {
      r -= dir_dr(d);
      cc -= dir_dc(d);
      if (r < 0 || r >= v.h || cc < 0 || cc >= v.w) break;
      const int q = r * v.w + cc;
      if (v.wall[q]) break;
      if (v.fuse[q] > 0) {
        if (k <= blast_of(v, q, default_blast)) best = fmaxf(best, val[q]);
        break;
      }
      if (v.brick[q]) break;
    }
  }
  return best;
}

// Per-warp scratch for the danger map, indexed by cell.
struct DangerScratch {
  float* cur;     // chain-corrected bomb weights
  float* front;   // front value (0 = not in front)
  float* spread;
  uint16_t* bombs;
};

// Stage A (chain correction among bombs, sim/blast.py:251-289).  Fills
// s.cur[c] for every bomb cell (other entries are not written).  Returns the
// bomb count.
// Each round is a scatter: lane (front bomb, direction) walks its ray up to
// its blast and raises the first bomb it meets (walls stop it, bricks end
// it) with the front value.  That is the reference's front propagation,
// which shifts each front bomb's value outwards and masks it with the
// passability of the cell it lands on, never of the cell it starts from: a
// bomb on a wall cell (a player standing on an obstacle can place one) is a
// source here as there, and never a target.
// nb_known >= 0: s.bombs already holds the nb_known bomb cells.
// wtab (optional): fuse_weight(f, fuse_f) for f = 0..31, read instead of
// dividing for fuses below 32 (the same values).
__device__ inline int danger_stage_a(const Env& v, const DangerScratch& s, float fuse_f,
                                     int default_blast, int rounds, int* max_b_out,
                                     int nb_known = -1, const float* wtab = nullptr) {
  const int lane = lane_id();
  const int nb = nb_known >= 0 ? nb_known
                               : warp_compact(v.cells, s.bombs, [&](int c) { return v.fuse[c] > 0; });
  // only bomb entries of cur / front are ever read (here, by the paint and
  // by danger_at), so the weights are computed for the bombs alone
  int mb = 0;
  for (int i = lane; i < nb; i += 32) {
    const int c = s.bombs[i];
    const int f = v.fuse[c];
    const float w = (wtab && f >= 0 && f < 32) ? wtab[f] : fuse_weight(f, fuse_f);
    s.cur[c] = w;
    s.front[c] = w;
    mb = max(mb, blast_of(v, c, default_blast));
  }
  mb = warp_max(mb);
  *max_b_out = mb;
  __syncwarp();
  for (int r = 0; r < rounds && nb > 0; ++r) {
    for (int i = lane; i < nb; i += 32) s.spread[s.bombs[i]] = 0.f;
    __syncwarp();
    for (int i = lane; i < 4 * nb; i += 32) {
      const int f = s.bombs[i >> 2], d = i & 3;
      const float fv = s.front[f];
      if (!(fv > 0.f)) continue;
      const int bl = blast_of(v, f, default_blast);
      int rr = f / v.w, cc = f - rr * v.w;
      for (int k = 1; k <= bl; ++k) {
        rr += dir_dr(d);
        cc += dir_dc(d);
        if (rr < 0 || rr >= v.h || cc < 0 || cc >= v.w) break;
        const int c = rr * v.w + cc;
        if (v.wall[c]) break;
        if (v.fuse[c] > 0) {
          atomicMax(reinterpret_cast<int*>(s.spread + c), __float_as_int(fv));
          break;
        }
        if (v.brick[c]) break;
      }
    }
    __syncwarp();
    // each bomb is updated by one lane and reads only its own entries here
    bool any_new = false;
    for (int i = lane; i < nb; i += 32) {
      const int c = s.bombs[i];
      const float sp = s.spread[c];
      const bool nw = sp > s.cur[c];
      s.cur[c] = fmaxf(s.cur[c], sp);
      s.front[c] = nw ? sp : 0.f;   // newly raised bombs form the next front
      any_new |= nw;
    }
    __syncwarp();
    if (!__any_sync(QQT_FULL, any_new)) break;
  }
  return nb;
}

// Stage B value at one cell (sim/blast.py:291-317): walls 0, else the max of
// the cell's own bomb weight and every reaching bomb's corrected weight.
__device__ __forceinline__ float danger_at(const Env& v, const DangerScratch& s, int c,
                                           int default_blast, int max_b) {
  if (v.wall[c]) return 0.f;
  const float own = v.fuse[c] > 0 ? s.cur[c] : 0.f;
  return fmaxf(own, reach_max(v, c, s.cur, default_blast, max_b));
}

// danger_at for every player at once (warp-wide): lane 4 p + d walks
// direction d from player p's cell `cell` (lane p's value), the four lanes
// of a player combine by max (exact, so the same value as danger_at), and
// lane p (p < P) returns the player's danger; other lanes return 0.
__device__ inline float danger_at_players(const Env& v, const DangerScratch& s, int cell,
                                          int default_blast, int max_b, int P) {
  const int lane = lane_id();
  const int p = lane >> 2, d = lane & 3;
  const int c = __shfl_sync(QQT_FULL, cell, p);
  float best = 0.f;
  if (p < P) {
    const int r0 = c / v.w, c0 = c - r0 * v.w;
    int r = r0, cc = c0;
    for (int k = 1; k <= max_b; ++k) {
      r -= dir_dr(d);
      cc -= dir_dc(d);
      if (r < 0 || r >= v.h || cc < 0 || cc >= v.w) break;
      const int q = r * v.w + cc;
      if (v.wall[q]) break;
      if (v.fuse[q] > 0) {
        if (k <= blast_of(v, q, default_blast)) best = s.cur[q];
        break;
      }
      if (v.brick[q]) break;
    }
  }
  best = fmaxf(best, __shfl_xor_sync(QQT_FULL, best, 1));
  best = fmaxf(best, __shfl_xor_sync(QQT_FULL, best, 2));
  const float reach = __shfl_sync(QQT_FULL, best, (4 * lane) & 31);
  if (lane >= P || v.wall[cell]) return 0.f;
  const float own = v.fuse[cell] > 0 ? s.cur[cell] : 0.f;
  return fmaxf(own, reach);
}

// Stage B for a whole env (sim/blast.py:291-317), scatter form: out[c] =
// the cell's own bomb weight (0 elsewhere, walls 0), raised by every bomb's
// corrected weight along its four rays.  Lane (bomb, direction) walks
// k = 1..blast(bomb) cells outwards: a wall stops the ray before it, any
// other cell is raised (shared-memory atomicMax on the bits of the
// non-negative float), and a bomb or brick stops the ray after it.  A cell
// thus receives exactly the bombs it would find as the first solid cell
// within their blast when looking along each direction: the same set, and
// max is exact, so the values are identical to the gather form.  The
// reference spreads the weights with walls zeroed (seed = weight *
// passable), so a bomb on a wall cell casts no rays here, and wall cells
// stay 0.
__device__ inline void danger_paint(const Env& v, const DangerScratch& s, int nb,
                                    int default_blast, float* out) {
  const int lane = lane_id();
#pragma unroll
  for (int c = lane; c < v.cells; c += 32)
    out[c] = (v.fuse[c] > 0 && !v.wall[c]) ? s.cur[c] : 0.f;
  __syncwarp();
  for (int i = lane; i < 4 * nb; i += 32) {
    const int q = s.bombs[i >> 2], d = i & 3;
    const float val = s.cur[q];
    if (!(val > 0.f) || v.wall[q]) continue;
    const int bl = blast_of(v, q, default_blast);
    int r = q / v.w, cc = q - r * v.w;
    for (int k = 1; k <= bl; ++k) {
      r += dir_dr(d);
      cc += dir_dc(d);
      if (r < 0 || r >= v.h || cc < 0 || cc >= v.w) break;
      const int c = r * v.w + cc;
      if (v.wall[c]) break;
      atomicMax(reinterpret_cast<int*>(out + c), __float_as_int(val));
      if (v.fuse[c] > 0 || v.brick[c]) break;
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------ movement

// Either of two cells blocks a player whose box currently spans
// rows [ra, rb] x cols [ca, cb] (sim/move.py:72-95).
__device__ __forceinline__ bool impassable_pair(const Env& v, int r0, int c0, int r1, int c1,
                                                int ra, int rb, int ca, int cb) {
  const int h = v.h, w = v.w;
  if (r0 < 0 || r0 >= h || c0 < 0 || c0 >= w || r1 < 0 || r1 >= h || c1 < 0 || c1 >= w)
    return true;
  const int q0 = r0 * w + c0, q1 = r1 * w + c1;
  const bool s0 = v.wall[q0] || v.brick[q0] || v.fuse[q0] > 0;
  const bool s1 = v.wall[q1] || v.brick[q1] || v.fuse[q1] > 0;
  const bool in0 = r0 >= ra && r0 <= rb && c0 >= ca && c0 <= cb;
  const bool in1 = r1 >= ra && r1 <= rb && c1 >= ca && c1 <= cb;
  return (s0 && !in0) || (s1 && !in1);
}

// Slide along one axis; stop flush against the first blocking cell
// (sim/move.py:98-151).  Same float operation order as the reference.
__device__ inline float resolve_axis(const Env& v, float coord, float delta, float other,
                                     float y, float x, float rad, bool vertical) {
  const float sgn = delta > 0.f ? 1.f : (delta < 0.f ? -1.f : 0.f);
  const float sr = __fmul_rn(sgn, rad);
  const int old_lead = (int)floorf(__fadd_rn(__fsub_rn(coord, delta), sr));
  const int new_lead = (int)floorf(__fadd_rn(coord, sr));
  const int lo = min(old_lead, new_lead), hi = max(old_lead, new_lead);
  const int span0 = (int)floorf(__fsub_rn(other, rad));
  const int span1 = (int)floorf(__fadd_rn(other, rad));
  const int ra = (int)floorf(__fsub_rn(y, rad)), rb = (int)floorf(__fadd_rn(y, rad));
  const int ca = (int)floorf(__fsub_rn(x, rad)), cb = (int)floorf(__fadd_rn(x, rad));
  // the two cells of each probed line: (lead, span0) / (lead, span1) moving
  // vertically, (span0, lead) / (span1, lead) horizontally; selected rather
  // than branched, so lanes probing different axes do not diverge
  const int lo_r0 = vertical ? lo : span0, lo_c0 = vertical ? span0 : lo;
  const int lo_r1 = vertical ? lo : span1, lo_c1 = vertical ? span1 : lo;
  const int hi_r0 = vertical ? hi : span0, hi_c0 = vertical ? span0 : hi;
  const int hi_r1 = vertical ? hi : span1, hi_c1 = vertical ? span1 : hi;
  const bool hit_lo = impassable_pair(v, lo_r0, lo_c0, lo_r1, lo_c1, ra, rb, ca, cb);
  const bool hit_hi = impassable_pair(v, hi_r0, hi_c0, hi_r1, hi_c1, ra, rb, ca, cb);
  const bool pos = sgn > 0.f;
  const int first_lead = pos ? hi : lo, second_lead = pos ? lo : hi;
  const bool first_hit = pos ? hit_hi : hit_lo, second_hit = pos ? hit_lo : hit_hi;
  if (!(first_hit || second_hit)) return coord;
  const float f = (float)(first_hit ? first_lead : second_lead);
  const float eps = 1e-4f;
  return pos ? __fsub_rn(__fsub_rn(f, rad), eps)
             : __fadd_rn(__fadd_rn(__fadd_rn(f, 1.f), rad), eps);
}

// Centre cell of a position, clamped to the grid (sim/move.py:282-288 plus
// the reference's defensive clamp); out-of-grid positions raise a flag.
__device__ __forceinline__ int center_cell(float y, float x, int h, int w) {
  const int r = (int)floorf(y), c = (int)floorf(x);
  int flat = r * w + c;
  if (r < 0 || r >= h || c < 0 || c >= w) {
    flag_error(QQT_DEV_POS_RANGE);
    flat = min(max(flat, 0), h * w - 1);
  }
  return flat;
}

// Deterministic uniform in [0, 1) from a 64-bit key (splitmix64 finaliser).
__host__ __device__ __forceinline__ float hash_uniform(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (float)(x >> 40) * (1.0f / 16777216.0f);
}

// The top 24 bits of the same finaliser, as an integer.
__host__ __device__ __forceinline__ uint32_t hash_u24(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (uint32_t)(x >> 40);
}

}  // namespace qqt

static inline int check_cfg(const QqtCfg* cfg) {
  if (!cfg) return QQT_E_ARG;
  if (cfg->n_envs <= 0 || cfg->height <= 0 || cfg->width <= 0) return QQT_E_ARG;
  if (cfg->height > QQT_MAX_H || cfg->width > QQT_MAX_W || cfg->n_players < 2 ||
      cfg->n_players > QQT_MAX_P)
    return QQT_E_LIMIT;
  return QQT_OK;
}

// SM count of the current device (cached per device; host threads may
// race to fill an entry, and all of them store the same value).
static inline int sm_count() {
  static std::atomic<int> n[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int v = n[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

static inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? QQT_OK : QQT_E_LAUNCH;
}
