/*
 * qqt_b200.h -- C ABI of the B200 rollout engine (libqqt_b200.so).
 *
 * Drop-in boundary for the reference's batched simulator path: each entry
 * point replaces one reference call (cited per function).  The reference is
 * Python, so its natural binding is ctypes; INTEGRATION.md shows the stub.
 *
 * Conventions
 *   - All pointers are device pointers owned by the caller.  The library
 *     never allocates or frees device memory and keeps no pointer across
 *     calls (the MLP weight pack is a caller-owned buffer too).
 *   - Every call is stream-ordered on `stream` and does not synchronise the
 *     host, so a whole rollout tick can be captured into one CUDA graph.
 *   - Return value: QQT_OK (0) or a QQT_E_* code for argument errors and
 *     launch failures.  Conditions detected inside kernels (out-of-range
 *     positions, relaxation not converged) are OR-ed into a device error
 *     word that qqt_get_error() reads and clears.
 *
 * Layout (N envs, C = H*W cells, P players):
 *   plane   [N][C]       wall/brick/crate/recycle (uint8 0/1), fuse (int16),
 *                        owner (int8), bomb_blast (int16); env-major, the
 *                        reference's (N, H, W) tensors as they are
 *   player  [P][N]       alive/hp (uint8), since_bomb (int32),
 *                        bombs_cap/blast_cap/invuln/pending_lost/combo/
 *                        last_hit/lo_bombs/lo_blast (int64),
 *                        spd_g/lo_spd (float)
 *   pos     [P][2][N]    float (row, col) of each player's centre
 *   env     [N]          t (int64), crate_prob (float), hazard (uint8)
 *   obs     [N][obs_stride] fp16 (or fp32), channel-major (C_obs, H, W) per
 *                        env, rows padded to obs_stride elements (16 bytes
 *                        multiple) with zeros
 *   masks   move [N][P][5], bomb [N][P][2] uint8
 *   actions [N][P][2] int64 (move, bomb)
 */
#ifndef QQT_B200_H
#define QQT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qqt_stream_t;   /* == cudaStream_t */

enum {
  QQT_OK = 0,
  QQT_E_ARG = 1,         /* null pointer, bad size or unsupported config     */
  QQT_E_ALIGN = 2,       /* pointer or stride misaligned                     */
  QQT_E_LIMIT = 3,       /* N, H, W or P above the compiled limits            */
  QQT_E_LAUNCH = 4,      /* CUDA launch error                                 */
  QQT_E_DEVICE = 5       /* unsupported device (needs sm_100)                 */
};

/* device error word bits (qqt_get_error) */
enum {
  QQT_DEV_POS_RANGE = 1u << 0,   /* a centre cell fell outside the grid     */
  QQT_DEV_NOT_CONVERGED = 1u << 1, /* path-field relaxation hit its cap     */
  QQT_DEV_BAD_ACTION = 1u << 2,  /* action index outside its head's range   */
  QQT_DEV_TIMEOUT = 1u << 3,     /* a bounded mbarrier wait expired         */
  QQT_DEV_BAD_INDEX = 1u << 4    /* a gather index outside its source rows  */
};

/* Scalar configuration.  Float fields hold the float32 values the reference
 * multiplies by (products of Python doubles are formed in double, then
 * rounded once), so results match bit for bit.  Mirrors sim/config.py:102-603
 * plus the derived quantities the kernels need. */
typedef struct QqtCfg {
  int32_t n_envs, height, width, n_players;
  int32_t fuse, blast, max_steps, invuln_ticks, max_hp;
  int32_t resolve_rounds;   /* min(max_chain-1, chain_cap_rounds)             */
  int32_t danger_rounds;    /* min(max_chain, chain_cap_rounds), 0 if max_chain<=1 */
  int32_t corridor;         /* map_mode == "corridor": crates and growth      */
  int32_t hit_attr_penalty, growth_bombs_max, growth_blast_max;
  int32_t place_dist_cooldown, crate_speed_only, timeout_draw, win_hp_scaled;
  int32_t combo_on, obs_extra, obs_channels, obs_stride, obs_fp32;
  float radius, step_len, move_eps2;   /* move_eps2 = 2e-4                    */
  float step_penalty, hit_reward, brick_reward, danger_penalty; /* coef*dp   */
  float explore_coef, place_cover_reward, place_chain_reward, place_dist_reward;
  float place_dist_radius, chain_time_factor, chain_time_rest; /* 1-cf       */
  float growth_speed_step, growth_speed_max, pen_speed; /* pen*step         */
  float recycle_crate_prob, combo_reward, combo_gap_factor, win_bonus;
  float win_bonus_per_hp, chain_blast_bonus, obs_growth_bombs_max;
  float fuse_f, max_steps_f, h_minus_rad, w_minus_rad;
  /* hazard waves (sim/torch_sim.py:1404-1466): in envs with state hazard
   * set, every hazard_wave_ticks ticks (t > 0, t counted after the step's
   * increment) hazard_bombs_min..max bombs land on free cells with blast
   * drawn from hazard_blast_min..max, biased upwards as t approaches
   * hazard_ramp_ticks (= ramp seconds x tick_hz).  Draws are counter-based
   * hashes of (hazard_seed, env, t), not the reference's torch generator. */
  int32_t hazard_on, hazard_wave_ticks, hazard_bombs_min, hazard_bombs_max;
  int32_t hazard_blast_min, hazard_blast_max;
  float hazard_ramp_ticks;
  uint32_t hazard_seed_lo, hazard_seed_hi;
} QqtCfg;

typedef struct QqtState {
  uint8_t *wall, *brick, *crate, *recycle;
  int16_t *fuse;
  int8_t *owner;
  int16_t *bomb_blast;
  float *pos;
  uint8_t *alive, *hp;
  int32_t *since_bomb;
  int64_t *t;
  int64_t *bombs_cap, *blast_cap;
  float *spd_g;
  int64_t *invuln, *pending_lost, *combo, *last_hit, *lo_bombs, *lo_blast;
  float *lo_spd, *crate_prob;
  uint8_t *hazard;
} QqtState;

/* Per-env reset template used by the device-side auto-reset (the
 * benchmark configurations reset every env to its own template map; see
 * qqt_step).  Planes [N][C]; caps [P][N]; spawn [P][2][N]. */
typedef struct QqtTemplate {
  const uint8_t *wall, *brick, *crate;
  const float *spawn;
  const int64_t *bombs_cap, *blast_cap;
  const float *spd;
  const float *crate_prob;
  uint64_t seed;            /* spawn-swap draws: hash(seed, env, episode)     */
  int32_t swap_spawns;      /* 1: swap P0/P1 spawns with probability 1/2     */
  int32_t since_bomb0;      /* place_dist_cooldown                            */
  int64_t *episode;         /* [N] per-env reset counter (in/out)             */
} QqtTemplate;

/* Per-episode level generation on the device: the reference's reset_
 * (sim/torch_sim.py:178-420 with sim/mapgen.py's make_walls, make_bricks,
 * make_open_obstacles, make_ring_walls, make_ring_bricks).  The geometry
 * that does not change between episodes comes precomputed from the host
 * (cell bit sets, spawn positions, thresholds); the random parts are drawn
 * from a counter-based hash of (seed, env, episode, draw family, index)
 * instead of the host generator, so an ended episode's next level is built
 * with no host round trip.  Bit sets: bit c of word c / 32 = cell c. */
#define QQT_MG_WORDS 14           /* ceil(21 * 21 / 32)                        */
typedef struct QqtMapGen {
  uint64_t seed;
  int64_t *episode;               /* [N] per-env reset counter (in/out)        */
  const int64_t *opp_boost;       /* [N] opponent start tier 0/1/2 or NULL (0) */
  uint8_t *is_open;               /* [N] out, or NULL                          */
  int64_t *map_kind;              /* [N] out (0 corridor, 1 open, 2 ring), or NULL */
  int32_t corridor_mode;          /* map_mode == "corridor"; else an open map  */
  float cut_pure, cut_open, cut_ring; /* float32 kind thresholds: pure_open,
                                     + open_fraction, + ring_fraction          */
  int32_t obst_max;               /* open_obstacle_max                         */
  int32_t random_wall_rows, top_wall_rows, corr_c0, corr_c1;
  int32_t n_edge, edge_cols[4];   /* columns of the vertical brick segments    */
  float wall_density, ring_density, hazard_fraction;
  int32_t ring_r0, ring_r1, ring_c0, ring_c1; /* central block [r0,r1)x[c0,c1) */
  int32_t open_cross;             /* open maps get the cross-band crates       */
  /* seat-0 start attributes by level kind: [0] corridor / ring (growth
   * start), [1] open and pure-open maps, [2] open-mode maps */
  int64_t start_bombs[3], start_blast[3];
  float start_spd[3];
  float crate_prob_kind[3];       /* corridor, open, ring                      */
  int64_t opp_bombs2, opp_blast2; /* opponent tier 2 start                     */
  float opp_spd2, opp_mult;       /* tier 2 speed; tier 1 multiplier           */
  int64_t bombs_max, blast_max;   /* growth caps (tier 1 clamp)                */
  float spd_max;
  float spawn[3][4][2];           /* [map spawns, open spawns, ring spawns][player][row, col] */
  uint32_t clear_spawn[QQT_MG_WORDS]; /* map spawn cells + 4-neighbours        */
  uint32_t clear_ring[QQT_MG_WORDS];  /* ring spawn cells + 4-neighbours       */
  uint32_t cross[QQT_MG_WORDS];       /* open-map cross-band crate cells       */
} QqtMapGen;

/* Optional outputs of a step (any may be NULL). */
typedef struct QqtStepOut {
  float *reward;            /* [N][P]                                         */
  uint8_t *done;            /* [N]                                            */
  uint8_t *died, *winner;   /* [N][P]                                         */
  int64_t *n_alive;         /* [N]                                            */
  uint8_t *covered, *triggered; /* [N][C]                                     */
  uint8_t *reset_mask;      /* [N] envs reset by the device auto-reset        */
  uint8_t *hit;             /* [N][P] lost hp this tick in an env that did not
                               end: the rollout's damage flag, (hp before the
                               step - hp after the auto-reset step) > 0
                               (train/ppo.py:247-251); may be NULL           */
} QqtStepOut;

/* One tick of the environment, fused: fuse countdown, sequential bomb
 * placement, placement bonus, AABB sliding, chain explosion, bricks to
 * crates, damage, clearing, rewards (step/hit/place/attribute penalty/crate
 * pickup and growth/danger standing/combo/terminal) and done.
 * Replaces BatchedSim.step (sim/torch_sim.py:895-1261).
 *   actions   [N][P][2] int64
 *   rb_hit, rb_grow  [N][P] float uniforms for crate pickup (the reference's
 *             `_rand_buf` halves, sim/torch_sim.py:1129-1138); may be NULL
 *             when cfg->corridor == 0
 *   tiers     device int32: the blast tiers the chain resolver considers.
 *             The reference fixes them on its first step
 *             (sim/torch_sim.py:818-832); with first_step != 0 the call
 *             records max(bomb_blast.max() after placement, blast) into
 *             *tiers (two launches: placement, then the rest), later calls
 *             read it.
 *   scratch   device buffer of qqt_step_scratch_bytes(cfg) bytes
 *   tmpl      NULL: no reset (the caller resets on the host);
 *             otherwise done envs are reset on the device to their template.
 */
int qqt_step(const QqtCfg *cfg, const QqtState *st, const int64_t *actions,
             const float *rb_hit, const float *rb_grow, int32_t *tiers,
             int32_t first_step, const QqtStepOut *out, const QqtTemplate *tmpl,
             void *scratch, qqt_stream_t stream);
uint64_t qqt_step_scratch_bytes(const QqtCfg *cfg);

/* qqt_step fused with the next tick's observation: after the step (and the
 * device auto-reset) the same kernel writes the observation row and legal
 * masks of the resulting state, exactly what qqt_observe would produce for
 * it (the danger map reuses the step's danger-standing computation).
 * Replaces BatchedSim.step followed by the next tick's observe() +
 * legal_mask() in SelfPlayRunner.collect (train/ppo.py:215-249).
 *   obs  [N][obs_stride] fp16 rows (cfg->obs_fp32 must be 0), 16-byte
 *        aligned, obs_stride % 8 == 0;  mm [N][P][5], bm [N][P][2] uint8.
 *   obs_tiles  NULL, or [N][4] uint32 (16-byte aligned): row e's K-tile
 *        flags for qqt_mlp_act -- K tile t (row entries [64 t, 64 t + 64))
 *        holds a nonzero only if bit min(t >> 2, 31) of word t & 3 is set.
 * Other arguments as qqt_step. */
int qqt_step_observe(const QqtCfg *cfg, const QqtState *st, const int64_t *actions,
                     const float *rb_hit, const float *rb_grow, int32_t *tiers,
                     int32_t first_step, const QqtStepOut *out, const QqtTemplate *tmpl,
                     void *scratch, void *obs, uint8_t *mm, uint8_t *bm, uint32_t *obs_tiles,
                     qqt_stream_t stream);

/* qqt_step for callers that cannot allocate device memory (for example code
 * running inside another runtime's stream capture, or an embedding that only
 * hands this library pre-placed buffers).  No counterpart in the reference:
 * it exists only for such callers.  Same arguments and results as qqt_step
 * minus `scratch`: the scratch lives in a static device array of
 * QQT_STEP_NOALLOC_MAX = 262144 bytes, so n_envs * n_players must not exceed
 * it (else QQT_E_LIMIT).  The array is held by every GPU that loads the
 * library until the process exits.  The first call on a device looks up the
 * array's device address with that device current; make that first call
 * before any stream capture.  All calls share the one array (the placement
 * flags of the first-step pass are written before they are read, so nothing
 * needs clearing): calls that overlap on the GPU race with each other.
 * Allocates nothing. */
int qqt_step_noalloc(const QqtCfg *cfg, const QqtState *st, const int64_t *actions,
                     const float *rb_hit, const float *rb_grow, int32_t *tiers,
                     int32_t first_step, const QqtStepOut *out, const QqtTemplate *tmpl,
                     qqt_stream_t stream);

/* Device auto-reset with per-episode level generation: every env whose
 * done[e] is set gets a new level and a fresh episode, as the reference's
 * reset_ gives it (sim/torch_sim.py:178-420; level kind by pure_open /
 * open / ring fractions, corridor walls with random top/bottom rows, side
 * bricks and edge segments, open-map obstacles and cross crates, ring
 * block and band bricks, start attributes with the opponent boost tier,
 * spawn swap, hazard envs), drawn from a counter-based hash of (seed, env,
 * episode) rather than the host generator.  Envs with done[e] = 0 are not
 * touched.  With obs (fp16 rows [N][obs_stride]), mm and bm non-NULL, the
 * reset envs' observation rows and legal masks are rewritten for the new
 * episode (after a qqt_step_observe, the rows of the envs that ended);
 * obs_tiles (may be NULL, layout of qqt_step_observe) then flags every K
 * tile of those rows.
 * The per-env counter mg->episode advances for every reset env. */
int qqt_map_reset(const QqtCfg *cfg, const QqtState *st, const QqtMapGen *mg,
                  const uint8_t *done, void *obs, uint8_t *mm, uint8_t *bm,
                  uint32_t *obs_tiles, qqt_stream_t stream);

/* Crate recycling on the device: for every player with pending lost
 * attribute layers, drop min(lost, free cells) crates on distinct free cells
 * (no wall, no brick, not in the exclusion set) chosen uniformly at random,
 * mark them recycled and clear the pending count.  Same rule as
 * BatchedSim.flush_recycle (sim/torch_sim.py:549-596), drawn from a
 * counter-based RNG keyed by (seed, counter, env, player) instead of the
 * host generator, so it needs no host round trip.
 *   excl_bits  host array of ceil(C/32) words, bit c = excluded cell c */
int qqt_flush_recycle(const QqtCfg *cfg, const QqtState *st, const uint32_t *excl_bits,
                      uint64_t seed, uint64_t counter, qqt_stream_t stream);

/* Danger map + shared observation + legal masks for the current state.
 * Replaces BatchedSim.observe (sim/torch_sim.py:605-627, encode_obs
 * sim/obs.py:48-136, danger_map sim/blast.py:158-317) and
 * BatchedSim.legal_mask (sim/torch_sim.py:636-645, sim/obs.py:170-229).
 *   obs     [N][obs_stride] fp16 (fp32 when cfg->obs_fp32); may be NULL
 *   danger  [N][C] float32 danger map; may be NULL
 *   mm, bm  [N][P][5], [N][P][2]; may be NULL */
int qqt_observe(const QqtCfg *cfg, const QqtState *st, void *obs, float *danger,
                uint8_t *mm, uint8_t *bm, qqt_stream_t stream);

/* Legal masks only (sim/obs.py:170-229). */
int qqt_legal_mask(const QqtCfg *cfg, const QqtState *st, uint8_t *mm, uint8_t *bm,
                   qqt_stream_t stream);

/* Bot entry points act for one seat.  Masks and actions are that seat's
 * rows: row e of the move mask starts at mm + e*mm_stride (5 entries), of
 * the bomb mask at bm + e*bm_stride (2 entries), of the action at
 * act + e*act_stride (move, bomb).  A slice mm[:, pid] of an [N][P][5] mask
 * is passed as (pointer to its first row, stride P*5). */

/* astar bot: own-bomb threat, the two shortest-path fields V_safe / V_opp
 * with cell cost 1 + 2*danger, candidate scoring, fallback and bomb
 * decision.  Replaces astar_attack + _mode_ticker (sim/bots.py:179-508,
 * 241-264).
 *   obs        [N][obs_stride] fp16 observation (danger channel is read)
 *   noise      [N][5] uniforms (the bot's torch.rand(n, 5))
 *   mode, timer [N] int64 mode-ticker state (NULL: always approach)
 *   tick16     1 when this call is a multiple-of-16 ticker call
 *   new_mode, new_timer [N] int64 draws used when a timer has expired on
 *              such a call (may be NULL when tick16 == 0)
 *   vsafe, vopp [N][C] float fields (may be NULL)
 *   scratch    >= 4 bytes of device memory (batch max of blast_cap[pid]) */
int qqt_astar_act(const QqtCfg *cfg, const QqtState *st, const void *obs,
                  const uint8_t *mm, int32_t mm_stride, const uint8_t *bm,
                  int32_t bm_stride, int32_t pid, const float *noise, int64_t *mode,
                  int64_t *timer, int32_t tick16, const int64_t *new_mode,
                  const int64_t *new_timer, int64_t *act, int32_t act_stride,
                  float *vsafe, float *vopp, void *scratch, qqt_stream_t stream);

/* hunter bot: the astar bot with the crate layer and no mode ticker
 * (make_bot "hunter" = astar_attack(eat_crates=True), sim/bots.py:557-561,
 * crate layer sim/bots.py:376-431).  With >= 2 of the seat's bomb / blast /
 * speed attributes under 70 % of their growth caps, a crate on the board
 * and the seat alive, it descends a third field V_crate (sources = crate
 * cells, the same cost and obstacles) unless escaping or no crate is
 * reachable.  Arguments as qqt_astar_act; vcrate [N][C] may be NULL. */
int qqt_hunter_act(const QqtCfg *cfg, const QqtState *st, const void *obs,
                   const uint8_t *mm, int32_t mm_stride, const uint8_t *bm,
                   int32_t bm_stride, int32_t pid, const float *noise, int64_t *act,
                   int32_t act_stride, float *vsafe, float *vopp, float *vcrate,
                   void *scratch, qqt_stream_t stream);

/* random bot (sim/bots.py:36-58): uniform legal move from u_move [N]
 * (inverse CDF over legal entries), bomb when u_bomb [N] < bomb_rate and
 * the bomb mask allows it. */
int qqt_random_act(const QqtCfg *cfg, const QqtState *st, const uint8_t *mm,
                   int32_t mm_stride, const uint8_t *bm, int32_t bm_stride, int32_t pid,
                   const float *u_move, const float *u_bomb, float bomb_rate,
                   int64_t *act, int32_t act_stride, qqt_stream_t stream);

/* greedy bot (sim/bots.py:95-176); noise [N][5] uniforms. */
int qqt_greedy_act(const QqtCfg *cfg, const QqtState *st, const void *obs,
                   const uint8_t *mm, int32_t mm_stride, const uint8_t *bm,
                   int32_t bm_stride, int32_t pid, const float *noise, int64_t *act,
                   int32_t act_stride, qqt_stream_t stream);

/* MLP policy (train/model.py:121-153, 167-245).  For each listed seat:
 * Linear(K -> 128) on the tensor cores (tcgen05 kind::f16, TMA-staged
 * operands, fp16 obs x the hi+lo fp16 halves of the seat-permuted fp32
 * weights, fp32 accumulation in TMEM; the seat's view permutation is folded
 * into the packed weights' column gather), then LN, ReLU, Linear(128,128),
 * LN, ReLU, the move/bomb/critic heads, masking with float32's lowest value
 * and inverse-CDF sampling a = #{k : u*S > cs_k} over exp(z - max z).
 * One kernel per 128 env rows: Linear(128,128) and the heads' hidden layer
 * also run on tcgen05 (fp16 hi/lo splits of activations and weights, three
 * products per K step), every intermediate stays in TMEM / shared memory.
 *   pack    weights packed by qqt_mlp_pack (256-byte aligned)
 *   obs     [N][obs_stride] fp16, obs_stride % 8 == 0, 16-byte aligned; the
 *           first k_in = C*H*W entries of each row are the observation
 *   obs_tiles  NULL (every K tile runs), or [N][4] uint32, 16-byte aligned:
 *           the rows' nonzero-K-tile flags as qqt_step_observe writes them.
 *           A K tile (64 entries) flagged in none of a 128-row tile's rows
 *           is skipped for those rows (it adds exactly zero); flags may
 *           over-report but must not miss a nonzero entry
 *   n_seats 1 or 2, the seats the pack was built for, in its order
 *   mm, bm  host arrays of n_seats device pointers: seat s's move-mask row e
 *           is at mm[s] + e*mm_stride (5 entries), bomb-mask row at
 *           bm[s] + e*bm_stride (2 entries)
 *   u       [n_seats][N][2] uniforms (move, bomb)
 *   act     host array of n_seats device pointers; row e of seat s at
 *           act[s] + e*act_stride (move, bomb int64)
 *   logp, value [n_seats][N] (may be NULL); logits [n_seats][N][8]
 *           (5 move, 2 bomb, value) or NULL
 *   work    reserved (may be NULL); qqt_mlp_work_bytes gives its size */
int qqt_mlp_act(const void *pack, const void *obs, const uint32_t *obs_tiles,
                int32_t n_envs, int32_t obs_stride,
                int32_t k_in, int32_t n_seats, const uint8_t *const *mm, int32_t mm_stride,
                const uint8_t *const *bm, int32_t bm_stride, const float *u,
                int64_t *const *act, int32_t act_stride, float *logp, float *value,
                float *logits, void *work, qqt_stream_t stream);
uint64_t qqt_mlp_work_bytes(int32_t n_envs, int32_t n_seats);

/* Pack the fp32 parameters of one ActorCritic(mlp) for qqt_mlp_act.
 * params: 20 device pointers in the order of qqt_mlp_param_names()
 * (the reference state_dict keys); pids[n_seats] (host) selects the view
 * permutations; pack: device buffer of qqt_mlp_pack_bytes() bytes, 256-byte
 * aligned.  Re-run after every optimizer step. */
int qqt_mlp_pack(const float *const *params, int32_t k_in, int32_t n_players,
                 int32_t channels, int32_t hw, int32_t n_seats, const int32_t *pids,
                 void *pack, qqt_stream_t stream);
uint64_t qqt_mlp_pack_bytes(int32_t k_in, int32_t n_seats);
const char *qqt_mlp_param_names(void);

/* CNN policy (train/model.py:77-101, 187-196): conv0 3x3 (C -> 16, the
 * seat's view permutation folded into its input channels) -> LN[16,H,W] ->
 * ReLU -> conv 16->32 -> LN -> ReLU -> conv 32->64 -> LN -> ReLU -> conv 1x1
 * 64->8 -> LN -> ReLU -> Linear(8HW->128), then the same tail as the MLP
 * (LN, ReLU, 128x128, LN, ReLU, heads, masking, inverse-CDF sampling).
 * Arguments as qqt_mlp_act; channels must be 14 (P = 2 layout);
 * work = qqt_cnn_work_bytes(N, n_seats). */
int qqt_cnn_act(const void *pack, const void *obs, int32_t n_envs, int32_t obs_stride,
                int32_t height, int32_t width, int32_t channels, int32_t n_seats,
                const uint8_t *const *mm, int32_t mm_stride, const uint8_t *const *bm,
                int32_t bm_stride, const float *u, int64_t *const *act, int32_t act_stride,
                float *logp, float *value, float *logits, void *work, qqt_stream_t stream);
uint64_t qqt_cnn_work_bytes(int32_t n_envs, int32_t n_seats);

/* Pack the fp32 parameters of one ActorCritic(cnn): params = 36 device
 * pointers in the order of qqt_cnn_param_names() (reference state_dict
 * keys); pids[n_seats] host array; pack = qqt_cnn_pack_bytes() bytes. */
int qqt_cnn_pack(const float *const *params, int32_t n_players, int32_t channels, int32_t hw,
                 int32_t n_seats, const int32_t *pids, void *pack, qqt_stream_t stream);
uint64_t qqt_cnn_pack_bytes(int32_t channels, int32_t hw, int32_t n_seats);
const char *qqt_cnn_param_names(void);

/* Generalised advantage estimation over a rollout buffer
 * (train/ppo.py:101-110): rew [T] rows of rew_stride floats (row t, env e
 * at rew[t*rew_stride + e]), done [T][N] uint8, val rows of val_stride,
 * last_val [N]; writes adv, ret [T][N] float32.  Same float32 operation
 * order as the reference loop. */
int qqt_gae(const float *rew, int32_t rew_stride, const uint8_t *done, const float *val,
            int32_t val_stride, const float *last_val, int32_t T, int32_t N, double gamma,
            double lam, float *adv, float *ret, qqt_stream_t stream);

/* Per-player features of the LSTM policy (sim/obs.py:241-340) from the
 * shared observation rows obs [N][obs_stride] (fp16, or fp32 with
 * obs_fp32): local [N][Po][C][7][7], rel [N][Po][10][6], glob [N][Po][5] in
 * the observation's dtype, Po = 1 with only_p0 else P.  max_bombs =
 * SimConfig.max_bombs.  Equal-distance bomb slots in ascending flat cell
 * order (the reference leaves that order to torch.topk). */
int qqt_local_view(const QqtCfg *cfg, const QqtState *st, const void *obs, int32_t max_bombs,
                   int32_t only_p0, void *local, void *rel, void *glob, qqt_stream_t stream);

/* ---- PPO update of the MLP policy: its first layer (train/ppo.py:364-437
 * via ActorCritic(mlp).evaluate, train/model.py:121-153 and 247-256).  The
 * reference runs `obs[sel]` (index gather), `.float()`, F.linear(x, W0[:,
 * inv_cols[pid]], b0) and autograd's weight gradient in float32 for every
 * minibatch; these entry points do the same from the float16 rows. */

/* dst row i = src row idx[i] (row_bytes of each; strides in bytes; all
 * 16-byte multiples).  An index outside [0, n_src) zero-fills its row and
 * raises QQT_DEV_BAD_INDEX. */
int qqt_gather_rows(const void *src, int64_t n_src, int64_t src_stride_bytes, const int64_t *idx,
                    int64_t n, void *dst, int64_t dst_stride_bytes, int64_t row_bytes,
                    qqt_stream_t stream);

/* W0 [128][k_in] float32 with seat pid's view permutation folded into its
 * column order (train/model.py:127-138), as fp16 hi then lo halves [2][128][kp]
 * (kp = k_in rounded up to 64); pack = qqt_l1_pack_bytes(k_in) bytes,
 * 256-byte aligned. */
int qqt_l1_pack(const float *w0, int32_t k_in, int32_t n_players, int32_t channels, int32_t hw,
                int32_t pid, void *pack, qqt_stream_t stream);
uint64_t qqt_l1_pack_bytes(int32_t k_in);

/* h1 [n_rows][128] float32 = x W0p^T + b0 for fp16 rows x [n_rows][x_stride]
 * (x_stride >= k_in, a multiple of 8; columns >= k_in are not read). */
int qqt_l1_forward(const void *pack, const void *x, int64_t n_rows, int32_t x_stride,
                   int32_t k_in, const float *b0, float *h1, qqt_stream_t stream);

/* dw0 [128][k_in] float32 = dL/dW0 of the layer above for dL/dh1 = dh1
 * [n_rows][128] float32, in W0's own column order (seat pid's permutation
 * undone).  Row r of the input is x row r, or, with idx (n_rows int64 row
 * ids into x's n_src rows), x row idx[r] read in place (TMA gather4; an id
 * outside [0, n_src) reads row 0 and raises QQT_DEV_BAD_INDEX).  work =
 * qqt_l1_wgrad_work_bytes(n_rows, k_in) bytes, 1024-byte aligned. */
int qqt_l1_wgrad(const void *x, int64_t n_rows, int32_t x_stride, int32_t k_in,
                 const int64_t *idx, int64_t n_src, const float *dh1, int32_t n_players,
                 int32_t channels, int32_t hw, int32_t pid, float *dw0, void *work,
                 qqt_stream_t stream);
uint64_t qqt_l1_wgrad_work_bytes(int64_t n_rows, int32_t k_in);

/* Training forward of ActorCritic(mlp) for one seat (train/model.py:121-153,
 * 247-256): obs rows [n_rows][obs_stride] fp16 (or, with idx, row idx[r] of
 * obs's n_src rows, read in place by TMA gather4), legal masks, recorded
 * actions [n_rows][act_stride] int64 -> logp (of the actions), entropy, value
 * [n_rows] and the pre-LayerNorm activations h1, h2 [n_rows][128] that the
 * backward reads.  pack = qqt_mlp_pack(..., n_seats = 1, pids = {pid}, ...). */
int qqt_mlp_train_forward(const void *pack, const void *obs, int32_t n_rows, int32_t obs_stride,
                          int32_t k_in, const int64_t *idx, int64_t n_src, const uint8_t *mm,
                          int32_t mm_stride, const uint8_t *bm,
                          int32_t bm_stride, const int64_t *act, int32_t act_stride, float *logp,
                          float *ent, float *value, float *h1, float *h2, qqt_stream_t stream);

/* Backward of the layers above the first: g [3][n_rows] = dL/dlogp,
 * dL/dentropy, dL/dvalue per row -> grads[1..19] (device pointers in
 * qqt_mlp_param_names() order, reference shapes; grads[0], the first
 * layer's weight, comes from qqt_l1_wgrad on dh1) and dh1 = dL/dh1
 * [n_rows][128].  work = qqt_mlp_train_work_bytes(n_rows) bytes, 1024-byte
 * aligned. */
int qqt_mlp_train_backward(const void *pack, int32_t n_rows, int32_t k_in, const float *h1,
                           const float *h2, const uint8_t *mm, int32_t mm_stride,
                           const uint8_t *bm, int32_t bm_stride, const int64_t *act,
                           int32_t act_stride, const float *g, float *const *grads, float *dh1,
                           void *work, qqt_stream_t stream);
uint64_t qqt_mlp_train_work_bytes(int32_t n_rows);

/* Device error word: returns the accumulated QQT_DEV_* bits and clears
 * them (synchronises the device). */
int qqt_get_error(uint32_t *code_out);

/* Failure-path check of the policy kernel (no counterpart in the
 * reference, whose torch forward has no device-side waits).  With polls >
 * 0, every following launch of the fused MLP kernel (qqt_mlp_act, the
 * tail of qqt_cnn_act, qqt_mlp_train_forward) first makes one bounded
 * mbarrier wait of `polls` polls on a
 * barrier that nothing completes at that point, before any copy or MMA is
 * issued; the wait expires like any wait that runs out (QQT_DEV_TIMEOUT in
 * the error word) and the kernel takes its abort path: no outputs, TMEM
 * freed, every CTA of a cluster through the closing barrier.  polls = 0
 * (the default) turns the check off.  Host-global setting. */
int qqt_test_set_wait_polls(uint32_t polls);

/* Phase stamps (no counterpart in the reference).  A library built with
 * `build.py --phase-stamps` (libqqt_b200_phase.so) records, at the phase
 * boundaries of the step and MLP policy kernels, 16-byte records: word 0 =
 * kernel id << 56 | phase << 48 | SM << 32 | block << 8 | warp, word 1 =
 * the globaltimer in ns.  qqt_phase_read copies up to `cap` records to
 * host memory (n_out = the count) and qqt_phase_reset clears the ring.
 * The regular library returns QQT_E_ARG from both. */
int qqt_phase_read(uint64_t *host, uint32_t cap, uint32_t *n_out);
int qqt_phase_reset(void);

/* Library version string. */
const char *qqt_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QQT_B200_H */
