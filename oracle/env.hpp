// TEST INFRASTRUCTURE ONLY - the CPU oracle's environment layer (see nes.hpp for the usage rule).
//
// Restates, one env at a time:
//   * rl/csrc/controller.cuh:1-191  - move encoding, pad bytes, sticky restrict, legal masks, counter RNG, dropout;
//   * rl/csrc/reward10.cuh:546-632  - RewardTracker.update (double, Python evaluation order), parameterised by a
//     per-game spec so the synthetic games' seeded weights replace the reference constants
//     (rl/csrc/reward10_consts.h:24-35); the synthetic reader reads the template's RAM ($10-$17);
//   * rl/csrc/rlenv_core.cuh:138-414 - frame / render / finish / reset / restart / controls phases.
// Build with -ffp-contract=off: Python never fuses a*b+c (rl/csrc/reward10.cuh:1-6).
#pragma once
#include <cmath>
#include <cstdint>
#include <limits>
#include <vector>

#include "nes.hpp"

namespace orc {

// ------------------------------------------------------------------------------------------------ controller

namespace ctl {
constexpr int kMoves = 324, kDropInputs = 8, kTimeline = 45, kRing = 64, kDropMin = 8, kDropMax = 22;
constexpr u32 kGapP32 = 122713351u, kSticky32 = 0x40000000u;

struct Move { u8 dpad, a, b, start, select; };

inline u8 dpad_bits(int d) {
    static const u8 t[9] = {0, 0x10, 0x90, 0x80, 0xA0, 0x20, 0x60, 0x40, 0x50};
    return d >= 0 && d < 9 ? t[d] : 0;
}
inline int dpad_from_bits(u8 bits) { for (int d = 0; d < 9; ++d) if (dpad_bits(d) == bits) return d; return 0; }
inline int pack(Move m) { return m.dpad + 9 * (m.a + 3 * (m.b + 3 * (m.start + 2 * m.select))); }
inline Move unpack(int id) {
    Move m;
    m.dpad = static_cast<u8>(id % 9); id /= 9;
    m.a = static_cast<u8>(id % 3); id /= 3;
    m.b = static_cast<u8>(id % 3); id /= 3;
    m.start = static_cast<u8>(id % 2); id /= 2;
    m.select = static_cast<u8>(id % 2);
    return m;
}
inline u8 pad_byte(Move m, u64 frame) {
    const bool even = (frame & 1) == 0;
    u8 p = dpad_bits(m.dpad);
    if (m.a == 1 || (m.a == 2 && even)) p |= 1;
    if (m.b == 1 || (m.b == 2 && even)) p |= 2;
    if (m.start) p |= 8;
    if (m.select) p |= 4;
    return p;
}
inline Move restrict_move(Move m, int dropped, bool start_ok, bool select_ok) {
    u8 bits = dpad_bits(m.dpad);
    static const u8 dir[4] = {0x10, 0x20, 0x40, 0x80};
    if (dropped >= 0 && dropped < 4) bits &= static_cast<u8>(~dir[dropped]);
    m.dpad = static_cast<u8>(dpad_from_bits(bits));
    if ((dropped == 4 && m.a == 1) || (dropped == 6 && m.a == 2)) m.a = 0;
    if ((dropped == 5 && m.b == 1) || (dropped == 7 && m.b == 2)) m.b = 0;
    if (!start_ok) m.start = 0;
    if (!select_ok) m.select = 0;
    return m;
}
struct Masks { u16 dpad; u8 a, b, start, select; };
inline Masks legal(int dropped, bool start_ok, bool select_ok) {
    Masks k{0x1FF, 7, 7, static_cast<u8>(start_ok ? 3 : 1), static_cast<u8>(select_ok ? 3 : 1)};
    static const u8 dir[4] = {0x10, 0x20, 0x40, 0x80};
    if (dropped >= 0 && dropped < 4)
        for (int d = 0; d < 9; ++d) if (dpad_bits(d) & dir[dropped]) k.dpad &= static_cast<u16>(~(1u << d));
    if (dropped == 4) k.a &= ~2u;
    if (dropped == 6) k.a &= ~4u;
    if (dropped == 5) k.b &= ~2u;
    if (dropped == 7) k.b &= ~4u;
    return k;
}
inline u64 splitmix64(u64 x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
inline u32 rand_u32(u64 seed, u64& ctr) { return static_cast<u32>(splitmix64(seed ^ splitmix64(ctr++)) >> 32); }
inline u32 rand_below(u64 seed, u64& ctr, u32 n) { return static_cast<u32>((u64(rand_u32(seed, ctr)) * n) >> 32); }
inline u64 episode_seed(u64 run_seed, u32 env, u64 episode) {
    return splitmix64(splitmix64(run_seed ^ 0xD20F0D20F0ull) ^ (u64(env) << 40) ^ episode);
}

struct Dropout {
    u64 seed, counter;
    int32_t gap_left, drop_left, drop_input;
    u32 head;
    int8_t ring[kRing];
};
inline int32_t draw_gap(Dropout& s) { int32_t k = 1; while (rand_u32(s.seed, s.counter) >= kGapP32) ++k; return k; }
inline int8_t next_column(Dropout& s) {
    if (s.drop_left > 0) {
        const int8_t out = static_cast<int8_t>(s.drop_input);
        if (--s.drop_left == 0) s.gap_left = draw_gap(s);
        return out;
    }
    if (--s.gap_left == 0) {
        s.drop_input = static_cast<int32_t>(rand_below(s.seed, s.counter, kDropInputs));
        s.drop_left = kDropMin + static_cast<int32_t>(rand_below(s.seed, s.counter, kDropMax - kDropMin + 1));
    }
    return -1;
}
inline void dropout_reset(Dropout& s, u64 seed, bool enabled) {
    s.seed = seed; s.counter = 0; s.drop_left = 0; s.drop_input = -1; s.head = 0;
    s.gap_left = enabled ? draw_gap(s) : 0x7FFFFFFF;
    for (int j = 0; j < kRing; ++j) s.ring[j] = -1;
    for (int j = 0; j < kTimeline; ++j) s.ring[j] = enabled ? next_column(s) : -1;
}
inline int dropped_now(const Dropout& s) { return s.ring[s.head % kRing]; }
inline void dropout_advance(Dropout& s, bool enabled) {
    s.ring[s.head % kRing] = -1;
    ++s.head;
    s.ring[(s.head + kTimeline - 1) % kRing] = enabled ? next_column(s) : -1;
}
inline void timeline(const Dropout& s, u8* out) {
    for (int i = 0; i < kDropInputs * kTimeline; ++i) out[i] = 0;
    for (int j = 0; j < kTimeline; ++j) {
        const int b = s.ring[(s.head + j) % kRing];
        if (b >= 0) out[b * kTimeline + j] = 1;
    }
}
}  // namespace ctl

// ------------------------------------------------------------------------------------------------ reward10

namespace rw {
enum : u32 { kEvSkip = 1, kEvLevel = 2, kEvDeath = 4, kEvWon = 8, kEvGameOver = 16, kEvStall = 32, kEvRollback = 64 };
enum : u8 { kEndNone = 0, kEndGameOver = 1, kEndWon = 2, kEndSkip = 3, kEndStall = 4 };
constexpr int kParts = 7;

// Per-game parameters: the reference constants for a commercial game, seeded ones for a synthetic game.
// Field order = ghostrun-lab_b200/synth.py SPEC_FIELDS.
struct Spec {
    double progress_unit, score_unit, stall_frames, idle_per_frame, death_from_lives, start_ok, select_ok;
    double w_progress, w_level, w_death, w_damage, w_score, score_cap, score_level_budget, w_win, w_stall,
        w_rollback, rollback_drop, reader, frame_limit;
};
constexpr int kSpecFields = 20;

struct Signals {
    bool in_play; int level; double progress; bool progress_valid; bool dying;
    bool has_lives; int lives; bool has_health; double health; bool has_score; long long score;
    bool game_over, won;
};

struct EnvState {
    bool has_prev; Signals prev;
    bool has_best_level; int best_level;
    bool has_best_progress; double best_progress;
    int deaths; long long idle_frames; double score_used; bool done; u8 end_reason; bool overflow;
};

// The synthetic template's reader (ghostrun-lab_b200/synth.py RAM map).
inline Signals observe_synth(const u8* r) {
    Signals s{};
    const int mode = r[0x17];
    s.in_play = mode == 1;
    s.level = r[0x12];
    s.progress = static_cast<double>(r[0x10] | (r[0x11] << 8));
    s.progress_valid = mode == 1;
    s.dying = false;
    s.has_lives = true; s.lives = r[0x13];
    s.has_score = true;
    long long v = 0;
    for (int a = 0x14; a <= 0x16; ++a) v = v * 100 + (r[a] >> 4) * 10 + (r[a] & 15);
    s.score = v;
    s.game_over = mode == 2;
    s.won = false;
    return s;
}

struct Update { double reward; bool done; u32 events; int event_level; double part[kParts]; };

// RewardTracker.update (rl/csrc/reward10.cuh:546-632, scripts/reward10/reward.py:101-163) with the spec's weights.
inline Update update(const Spec& G, const u8* ram, int frames, EnvState& e) {
    const Signals s = observe_synth(ram);
    const bool has_p = e.has_prev;
    const Signals p = e.prev;
    double r = 0.0;
    u32 ev = 0;
    int ev_level = 0;
    bool fresh = false;
    e.has_prev = true;
    e.prev = s;
    Update out{0.0, true, 0u, 0, {}};
    double part[kParts] = {};
    if (e.done) return out;
    if (s.in_play) {
        if (!e.has_best_level) {
            e.has_best_level = true; e.best_level = s.level; e.has_best_progress = false; e.score_used = 0.0;
        } else if (s.level > e.best_level + 1) {
            ev |= kEvSkip; ev_level = s.level; e.done = true; e.end_reason = kEndSkip;
        } else if (s.level > e.best_level) {
            r += G.w_level; part[1] += G.w_level;
            ev |= kEvLevel; ev_level = s.level;
            e.best_level = s.level; e.has_best_progress = false; e.score_used = 0.0;
            fresh = true;
        }
        if (s.level == e.best_level && s.progress_valid) {
            if (!e.has_best_progress) {
                e.has_best_progress = true; e.best_progress = s.progress;
            } else if (s.progress > e.best_progress) {
                const double rp = G.w_progress * (s.progress - e.best_progress) / G.progress_unit;
                r += rp; part[0] += rp;
                e.best_progress = s.progress;
                fresh = true;
            }
        }
    }
    bool death = false;
    if (has_p) {
        if (G.death_from_lives == 0.0) death = s.dying && !p.dying;
        else death = s.has_lives && p.has_lives && s.lives < p.lives;
        if (death && (s.in_play || p.in_play)) {
            r += G.w_death; part[2] += G.w_death;
            e.deaths += 1;
            ev |= kEvDeath;
            fresh = true;
        }
        if (s.in_play && p.in_play && s.has_health && p.has_health && s.health < p.health) {
            const double rd = G.w_damage * (p.health - s.health);
            r += rd; part[3] += rd;
        }
        if (s.in_play && p.in_play && s.has_score && p.has_score && s.score > p.score) {
            double sr = G.w_score * static_cast<double>(s.score - p.score) / G.score_unit;
            if (G.score_cap < sr) sr = G.score_cap;
            const double left = G.score_level_budget - e.score_used;
            if (left < sr) sr = left;
            if (sr > 0) { r += sr; part[4] += sr; e.score_used += sr; }
        }
    }
    if (has_p && !e.done && !death && !s.dying && !p.dying && !s.won && !s.game_over && s.in_play && p.in_play &&
        s.progress_valid && p.progress_valid && s.level == p.level && s.level == e.best_level &&
        p.progress - s.progress >= G.rollback_drop * G.progress_unit) {
        r += G.w_rollback; part[6] += G.w_rollback;
        ev |= kEvRollback;
    }
    if (!fresh && !e.done && has_p && s.in_play && p.in_play && s.progress_valid && p.progress_valid &&
        s.progress <= p.progress) {
        const double ci = G.idle_per_frame * frames;
        r += ci; part[6] += ci;
    }
    e.idle_frames = (fresh || !has_p) ? 0 : e.idle_frames + frames;
    if (s.won) {
        r += G.w_win; part[5] += G.w_win;
        ev |= kEvWon; e.done = true; e.end_reason = kEndWon;
    } else if (s.game_over) {
        ev |= kEvGameOver; e.done = true; e.end_reason = kEndGameOver;
    } else if (!e.done && G.stall_frames >= 0.0 && static_cast<double>(e.idle_frames) >= G.stall_frames) {
        r += G.w_stall; part[6] += G.w_stall;
        ev |= kEvStall; e.done = true; e.end_reason = kEndStall;
    }
    out.reward = r; out.done = e.done; out.events = ev; out.event_level = ev_level;
    for (int k = 0; k < kParts; ++k) out.part[k] = part[k];
    return out;
}
}  // namespace rw

// ------------------------------------------------------------------------------------------------ env phases

constexpr int kFramesPerDecision = 4, kObsW = 240, kObsH = 224, kObsPixels = kObsW * kObsH;
constexpr int kMaskBytes = 19, kTimelineBytes = ctl::kDropInputs * ctl::kTimeline, kInfo = 8;
constexpr int kEndFault = 5, kEndLevelClear = 6, kEndFrameLimit = 7;

struct Game {
    Cart cart;
    rw::Spec spec;
    int game_id = 0;
    int n = 0, offset = 0;
    std::vector<Console> con;        // n consoles + the boot snapshot at [n]
    std::vector<Console> idle_snap;  // boot snapshot after k = 1..idle_tmpl idle frames
    u64 tmpl_target = 0;
    int idle_tmpl = 0;
    bool start_ok = false, select_ok = false;
    // Level starts (rl/csrc/rlenv_core.cuh GameCtx lv_*, rl/csrc/rlenv_build.hpp:212-252): lv_cap saved states,
    // slots < lv_levels are level entrances, the rest places. lv_deaths -1 = nothing saved; lv_claim = this
    // decision's best arrival (deaths << 32 | env), ~0 = none.
    int lv_cap = 0, lv_levels = 0;
    u32 lv_thresh = 0;
    bool lv_weighted = false;
    std::vector<Console> lv_con;
    std::vector<rw::EnvState> lv_st;
    std::vector<u64> lv_target;
    std::vector<u32> lv_frame;
    std::vector<int32_t> lv_deaths;
    std::vector<u64> lv_claim;
    std::vector<u32> lv_cdf;
};

struct Outputs {
    const int16_t* actions = nullptr;
    u8* obs = nullptr; u8* emph = nullptr; float* reward = nullptr; u8* done = nullptr; u8* masks = nullptr;
    u8* timeline = nullptr; u8* pads = nullptr; u32* events = nullptr; float* info = nullptr; float* parts = nullptr;
    int32_t* start_out = nullptr;    // ep_start of the episode that just ended (where done)
    int32_t* level_out = nullptr;    // level after the decision's update, -1 = not known yet
    float* progress_out = nullptr;   // within-level progress / progress_unit, NaN = not valid now
};

struct PerEnv {
    rw::EnvState st;
    ctl::Dropout drop;
    u64 target;
    u32 ep_frame;
    int16_t prev_applied;
    u64 sticky_seed, sticky_ctr;
    u32 episode;
    float ep_ret;
    int32_t ep_len, ep_maxlvl, ep_idle;
    u32 fault;
    u8 resetting;
};

struct World {
    std::vector<Game> games;
    std::vector<PerEnv> env;
    Outputs out;
    u64 run_seed = 0;
    int sticky = 1, idle_max = 0, dropout = 1, no_render = 0, episode_level_end = -1;
    int total = 0;
    std::vector<int32_t> ep_start;   // [total] slot each episode started from, -1 = power-on; empty = level starts off
};

inline void atomic_min_u64(u64* p, u64 v) {
    u64 cur = __atomic_load_n(p, __ATOMIC_RELAXED);
    while (v < cur && !__atomic_compare_exchange_n(p, &cur, v, true, __ATOMIC_RELAXED, __ATOMIC_RELAXED)) {}
}

inline void emu_frame(Game& g, PerEnv& pe, int e, u8 pad) {
    Console& m = g.con[e];
    m.pad = pad;
    if (pe.fault == 0) {
        const u32 f = step_until(g.cart, m, pe.target);
        if (f != 0) pe.fault = f;
    }
    pe.target += kFrameDots;
    ++pe.ep_frame;
}

inline void write_controls(const Game& g, World& w, int ge) {
    const PerEnv& pe = w.env[ge];
    const int d = ctl::dropped_now(pe.drop);
    const ctl::Masks k = ctl::legal(d, g.start_ok, g.select_ok);
    u8* m = w.out.masks + static_cast<u64>(ge) * kMaskBytes;
    for (int i = 0; i < 9; ++i) m[i] = (k.dpad >> i) & 1u;
    for (int i = 0; i < 3; ++i) m[9 + i] = (k.a >> i) & 1u;
    for (int i = 0; i < 3; ++i) m[12 + i] = (k.b >> i) & 1u;
    for (int i = 0; i < 2; ++i) m[15 + i] = (k.start >> i) & 1u;
    for (int i = 0; i < 2; ++i) m[17 + i] = (k.select >> i) & 1u;
    ctl::timeline(pe.drop, w.out.timeline + static_cast<u64>(ge) * kTimelineBytes);
}

// rl/csrc/rlenv_core.cuh:181-191
inline void ph_frame(Game& g, World& w, int e, int f) {
    const int ge = g.offset + e;
    PerEnv& pe = w.env[ge];
    ctl::Move m = ctl::unpack(w.out.actions[ge]);
    if (w.sticky && ctl::rand_u32(pe.sticky_seed, pe.sticky_ctr) < ctl::kSticky32)
        m = ctl::restrict_move(ctl::unpack(pe.prev_applied), ctl::dropped_now(pe.drop), g.start_ok, g.select_ok);
    pe.prev_applied = static_cast<int16_t>(ctl::pack(m));
    const u8 pad = ctl::pad_byte(m, pe.ep_frame);
    w.out.pads[static_cast<u64>(ge) * kFramesPerDecision + f] = pad;
    emu_frame(g, pe, e, pad);
}

// rl/csrc/rlenv_core.cuh:194-205
inline void ph_render(Game& g, World& w, int e, int f, bool restart_pass) {
    const int ge = g.offset + e;
    if (restart_pass && w.env[ge].resetting == 0) return;
    if (w.no_render) return;
    render_obs(g.cart, g.con[e], w.out.obs + (static_cast<u64>(ge) * kFramesPerDecision + f) * kObsPixels,
               w.out.emph + (static_cast<u64>(ge) * kFramesPerDecision + f) * kObsH);
}

// rl/csrc/rlenv_core.cuh:208-263: idle count, level-start coin and pick (drawn only when level starts are on),
// then the snapshot: a saved level start, the boot snapshot after k idle frames, or the boot snapshot.
inline void reset_state(Game& g, World& w, int e) {
    const int ge = g.offset + e;
    PerEnv& pe = w.env[ge];
    const u32 ep = ++pe.episode;
    const u64 seed = ctl::episode_seed(w.run_seed, static_cast<u32>(ge), ep);
    pe.sticky_seed = ctl::splitmix64(seed ^ 0x5717C4A55EEDull);
    pe.sticky_ctr = 0;
    int idle = 0;
    if (w.idle_max > 0) idle = static_cast<int>(ctl::rand_below(pe.sticky_seed, pe.sticky_ctr, static_cast<u32>(w.idle_max + 1)));
    int lv = -1;
    if (g.lv_cap > 0 && g.lv_thresh != 0 && ctl::rand_u32(pe.sticky_seed, pe.sticky_ctr) < g.lv_thresh) {
        u32 saved = 0;
        for (int s = 0; s < g.lv_cap; ++s) saved += g.lv_deaths[s] >= 0 ? 1u : 0u;
        if (g.lv_weighted) {
            const u32 u = ctl::rand_u32(pe.sticky_seed, pe.sticky_ctr);
            for (int s = 0; s < g.lv_cap && lv < 0; ++s)
                if (u < g.lv_cdf[s]) lv = s;
        } else if (saved > 0) {
            u32 pick = ctl::rand_below(pe.sticky_seed, pe.sticky_ctr, saved);
            for (int s = 0; s < g.lv_cap && lv < 0; ++s)
                if (g.lv_deaths[s] >= 0 && pick-- == 0) lv = s;
        }
    }
    const int k = lv < 0 && idle <= g.idle_tmpl ? idle : 0;
    if (lv >= 0) {
        g.con[e] = g.lv_con[lv];
        pe.target = g.lv_target[lv];
        pe.ep_frame = g.lv_frame[lv];
        pe.st = g.lv_st[lv];
    } else {
        g.con[e] = k == 0 ? g.con[g.n] : g.idle_snap[k - 1];
        pe.target = g.tmpl_target + static_cast<u64>(k) * kFrameDots;
        pe.ep_frame = static_cast<u32>(k);
        pe.st = rw::EnvState{};
    }
    if (!w.ep_start.empty()) w.ep_start[ge] = lv;
    pe.fault = 0;
    ctl::dropout_reset(pe.drop, seed, w.dropout != 0);
    pe.prev_applied = 0;
    pe.ep_idle = idle;
    pe.resetting = 1;
}

// rl/csrc/rlenv_core.cuh:266-309, plus the frame-limit end (reason 7) the synthetic specs ask for.
inline void ph_finish(Game& g, World& w, int e) {
    const int ge = g.offset + e;
    PerEnv& pe = w.env[ge];
    const rw::Update u = rw::update(g.spec, g.con[e].ram, kFramesPerDecision, pe.st);
    const bool faulted = pe.fault != 0;
    const bool level_clear = !u.done && !faulted && w.episode_level_end >= 0 && (u.events & rw::kEvLevel) != 0 &&
                             u.event_level == w.episode_level_end + 1;
    const bool frame_limit = !u.done && !faulted && !level_clear && g.spec.frame_limit > 0.0 &&
                             static_cast<double>(pe.ep_frame) >= g.spec.frame_limit;
    const bool done = u.done || faulted || level_clear || frame_limit;
    const float r = faulted ? 0.0f : static_cast<float>(u.reward);
    w.out.reward[ge] = r;
    if (w.out.parts)
        for (int k = 0; k < rw::kParts; ++k)
            w.out.parts[static_cast<u64>(ge) * rw::kParts + k] = faulted ? 0.0f : static_cast<float>(u.part[k]);
    w.out.done[ge] = done ? 1 : 0;
    w.out.events[ge] = u.events;
    pe.ep_ret += r;
    ++pe.ep_len;
    if (u.event_level > pe.ep_maxlvl) pe.ep_maxlvl = u.event_level;
    ctl::dropout_advance(pe.drop, w.dropout != 0);
    if (g.lv_cap > 0 && !done && (u.events & rw::kEvLevel) != 0 && u.event_level >= 0 && u.event_level < g.lv_levels) {
        const int d = pe.st.deaths < 0 ? 0 : pe.st.deaths;
        atomic_min_u64(&g.lv_claim[u.event_level], (static_cast<u64>(d) << 32) | static_cast<u32>(e));
    }
    if (w.out.level_out) w.out.level_out[ge] = pe.st.has_best_level ? pe.st.best_level : -1;
    if (w.out.progress_out)
        w.out.progress_out[ge] = pe.st.has_prev && pe.st.prev.progress_valid
            ? static_cast<float>(pe.st.prev.progress / g.spec.progress_unit) : std::numeric_limits<float>::quiet_NaN();
    if (done) {
        if (w.out.start_out) w.out.start_out[ge] = w.ep_start.empty() ? -1 : w.ep_start[ge];
        float* inf = w.out.info + static_cast<u64>(ge) * kInfo;
        inf[0] = pe.ep_ret;
        inf[1] = static_cast<float>(pe.ep_len);
        inf[2] = static_cast<float>(faulted ? kEndFault : level_clear ? kEndLevelClear
                                    : frame_limit ? kEndFrameLimit : pe.st.end_reason);
        inf[3] = static_cast<float>(pe.st.deaths);
        inf[4] = static_cast<float>(pe.ep_maxlvl);
        inf[5] = pe.st.overflow ? 1.0f : 0.0f;
        inf[6] = static_cast<float>(pe.ep_idle);
        inf[7] = static_cast<float>(pe.episode);
        reset_state(g, w, e);
    }
}

inline void ph_reset_idle(Game& g, World& w, int e) {
    PerEnv& pe = w.env[g.offset + e];
    if (!pe.resetting) return;
    const bool lv = !w.ep_start.empty() && w.ep_start[g.offset + e] >= 0;   // a level start emulates every idle frame
    const int done = !lv && pe.ep_idle <= g.idle_tmpl ? pe.ep_idle : 0;
    for (int i = done; i < pe.ep_idle; ++i) emu_frame(g, pe, e, 0);
}

inline void ph_reset_frame(Game& g, World& w, int e) {
    PerEnv& pe = w.env[g.offset + e];
    if (!pe.resetting) return;
    emu_frame(g, pe, e, 0);
}

inline void ph_reset_finish_controls(Game& g, World& w, int e) {
    const int ge = g.offset + e;
    PerEnv& pe = w.env[ge];
    if (pe.resetting) {
        (void)rw::update(g.spec, g.con[e].ram, pe.ep_idle + kFramesPerDecision, pe.st);
        pe.ep_ret = 0.0f;
        pe.ep_len = 0;
        const int sl = w.ep_start.empty() ? -1 : w.ep_start[ge];   // a place: its level is the tracker's
        pe.ep_maxlvl = sl >= g.lv_levels ? (pe.st.has_best_level ? pe.st.best_level : 0) : sl > 0 ? sl : 0;
        pe.resetting = 0;
    }
    write_controls(g, w, ge);
}

inline void restart_phases(Game& g, World& w, int e) {
    ph_reset_idle(g, w, e);
    for (int f = 0; f < kFramesPerDecision; ++f) {
        ph_reset_frame(g, w, e);
        ph_render(g, w, e, f, true);
    }
    ph_reset_finish_controls(g, w, e);
}

inline void env_start(Game& g, World& w, int e) { reset_state(g, w, e); restart_phases(g, w, e); }

inline void env_step(Game& g, World& w, int e) {
    for (int f = 0; f < kFramesPerDecision; ++f) {
        ph_frame(g, w, e, f);
        ph_render(g, w, e, f, false);
    }
    ph_finish(g, w, e);
    restart_phases(g, w, e);
}

// Level-start saves after every env's decision (rl/csrc/rlenv_core.cuh:344-387, order of rl/csrc/rlenv_cpu.cpp:
// 100-116): the claimed arrival replaces the saved one when nothing is saved yet or it died no more often.
inline void archive(Game& g, World& w) {
    for (int s = 0; s < g.lv_levels; ++s) {
        const u64 cl = g.lv_claim[s];
        if (cl == ~0ull) continue;
        const bool take = g.lv_deaths[s] < 0 || static_cast<int32_t>(cl >> 32) <= g.lv_deaths[s];
        if (take) {
            const int e = static_cast<int>(cl & 0xFFFFFFFFull);
            const PerEnv& pe = w.env[g.offset + e];
            g.lv_con[s] = g.con[e];
            g.lv_st[s] = pe.st;
            g.lv_target[s] = pe.target;
            g.lv_frame[s] = pe.ep_frame;
            g.lv_deaths[s] = static_cast<int32_t>(cl >> 32);
        }
        g.lv_claim[s] = ~0ull;
    }
}

// Place save (rl/places.py, rl/csrc/rlenv_core.cuh:366-375): env e's whole state into slot s >= lv_levels; the
// no-progress clock restarts.
inline void place_save(Game& g, World& w, int e, int s) {
    if (s < g.lv_levels || s >= g.lv_cap || e < 0 || e >= g.n) return;
    const PerEnv& pe = w.env[g.offset + e];
    g.lv_con[s] = g.con[e];
    g.lv_st[s] = pe.st;
    g.lv_st[s].idle_frames = 0;
    g.lv_target[s] = pe.target;
    g.lv_frame[s] = pe.ep_frame;
    g.lv_deaths[s] = 0;
}

}  // namespace orc
