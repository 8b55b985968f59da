// Decision semantics on the device: controller (moves, sticky repeats, dropout schedule), reward10, episode ends and
// restarts, and the kernels that run them. Behaviour follows rl/csrc/rlenv_core.cuh:138-414 (phases),
// rl/csrc/controller.cuh:41-187 (controller) and rl/csrc/reward10.cuh:546-632 (RewardTracker.update).
//
// Kernels of one decision (per game slice, one stream):
//   k_frames<B>(decision)  thread per env: 4 x (pad byte, one emulated frame into presentation slot f)
//   k_render<B>            warp per (env, frame): the 4 observations
//   k_finish               thread per env: reward, outputs, episode end -> restart from a snapshot record,
//                          restarting envs appended to a list; masks/timeline for the others
//   k_frames<B>(restart)   grid-stride over the list: idle frames + 4 neutral frames, first tracker update, controls
//   k_render<B>(list)      the restarted envs' first observation
// The reward arithmetic is double in Python's order; the library is built with -fmad=false (no fused a*b+c).
#pragma once
#include "render.cuh"

namespace gr {

// ------------------------------------------------------------------------------------------------ controller

__device__ __forceinline__ u32 dpad_bits(u32 d) {
    // 0 none, 1 Up, 2 Up-Right, 3 Right, 4 Down-Right, 5 Down, 6 Down-Left, 7 Left, 8 Up-Left
    // pad bits: 4 Up, 5 Down, 6 Left, 7 Right
    switch (d) {
        case 1: return 0x10u; case 2: return 0x90u; case 3: return 0x80u; case 4: return 0xA0u;
        case 5: return 0x20u; case 6: return 0x60u; case 7: return 0x40u; case 8: return 0x50u;
        default: return 0u;
    }
}
__device__ __forceinline__ u32 dpad_from_bits(u32 b) {
    for (u32 d = 0; d < 9; ++d) if (dpad_bits(d) == b) return d;
    return 0;
}
struct Move { u32 dpad, a, b, start, select; };
__device__ __forceinline__ Move unpack_move(int id) {
    Move m;
    m.dpad = id % 9; id /= 9;
    m.a = id % 3; id /= 3;
    m.b = id % 3; id /= 3;
    m.start = id % 2; id /= 2;
    m.select = id % 2;
    return m;
}
__device__ __forceinline__ int pack_move(Move m) {
    return static_cast<int>(m.dpad + 9 * (m.a + 3 * (m.b + 3 * (m.start + 2 * m.select))));
}
__device__ __forceinline__ u32 pad_byte(Move m, u64 frame) {
    const bool even = (frame & 1u) == 0;
    u32 p = dpad_bits(m.dpad);
    if (m.a == 1 || (m.a == 2 && even)) p |= 1u;
    if (m.b == 1 || (m.b == 2 && even)) p |= 2u;
    if (m.start) p |= 8u;
    if (m.select) p |= 4u;
    return p;
}
__device__ __forceinline__ Move restrict_move(Move m, int dropped, bool start_ok, bool select_ok) {
    u32 bits = dpad_bits(m.dpad);
    if (dropped >= 0 && dropped < 4) bits &= ~(0x10u << dropped);
    m.dpad = dpad_from_bits(bits);
    if ((dropped == 4 && m.a == 1) || (dropped == 6 && m.a == 2)) m.a = 0;
    if ((dropped == 5 && m.b == 1) || (dropped == 7 && m.b == 2)) m.b = 0;
    if (!start_ok) m.start = 0;
    if (!select_ok) m.select = 0;
    return m;
}
__device__ __forceinline__ u64 splitmix64(u64 x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__device__ __forceinline__ u32 rand_u32(u64 seed, u64& ctr) { return static_cast<u32>(splitmix64(seed ^ splitmix64(ctr++)) >> 32); }
__device__ __forceinline__ u32 rand_below(u64 seed, u64& ctr, u32 n) {
    return static_cast<u32>((static_cast<u64>(rand_u32(seed, ctr)) * n) >> 32);
}
constexpr u32 kGapP32 = 122713351u, kSticky32 = 0x40000000u;

__device__ __forceinline__ i32 draw_gap(Dropout& s) { i32 k = 1; while (rand_u32(s.seed, s.counter) >= kGapP32) ++k; return k; }
__device__ __forceinline__ int next_column(Dropout& s) {
    if (s.drop_left > 0) {
        const int out = s.drop_input;
        if (--s.drop_left == 0) s.gap_left = draw_gap(s);
        return out;
    }
    if (--s.gap_left == 0) {
        s.drop_input = static_cast<i32>(rand_below(s.seed, s.counter, kDropInputs));
        s.drop_left = 8 + static_cast<i32>(rand_below(s.seed, s.counter, 15));
    }
    return -1;
}
static __device__ void dropout_reset(Dropout& s, u64 seed, bool enabled) {
    s.seed = seed; s.counter = 0; s.drop_left = 0; s.drop_input = -1; s.head = 0;
    s.gap_left = enabled ? draw_gap(s) : 0x7FFFFFFF;
    for (int j = 0; j < kRing; ++j) s.ring[j] = -1;
    for (int j = 0; j < kTimeline; ++j) s.ring[j] = static_cast<int8_t>(enabled ? next_column(s) : -1);
}
__device__ __forceinline__ int dropped_now(const Dropout& s) { return s.ring[s.head % kRing]; }
static __device__ void dropout_advance(Dropout& s, bool enabled) {
    s.ring[s.head % kRing] = -1;
    ++s.head;
    s.ring[(s.head + kTimeline - 1) % kRing] = static_cast<int8_t>(enabled ? next_column(s) : -1);
}

// ------------------------------------------------------------------------------------------------ reward10

struct Sig {
    bool in_play, progress_valid, dying, has_lives, has_health, has_score, game_over, won;
    int level, lives;
    double progress, health;
    long long score;
};

// The synthetic template's RAM -> Signals ($10-$11 progress, $12 level, $13 lives, $14-$16 BCD score, $17 mode).
static __device__ Sig observe_synth(const StateView& S, u32 e) {
    const u32 w10 = S.ram[static_cast<u64>(0x10 >> 2) * S.Np + e];   // $10-$13
    const u32 w14 = S.ram[static_cast<u64>(0x14 >> 2) * S.Np + e];   // $14-$17
    Sig s;
    const u32 mode = w14 >> 24;
    s.in_play = mode == 1;
    s.level = static_cast<int>((w10 >> 16) & 0xFFu);
    s.progress = static_cast<double>(w10 & 0xFFFFu);
    s.progress_valid = mode == 1;
    s.dying = false;
    s.has_lives = true; s.lives = static_cast<int>(w10 >> 24);
    s.has_health = false; s.health = 0.0;
    s.has_score = true;
    long long v = 0;
    for (int k = 0; k < 3; ++k) { const u32 b = (w14 >> (8 * k)) & 0xFFu; v = v * 100 + (b >> 4) * 10 + (b & 15u); }
    s.score = v;
    s.game_over = mode == 2;
    s.won = false;
    return s;
}

struct Upd { double reward; bool done; u32 events; int event_level; double part[kParts]; };
enum : u32 { kEvSkip = 1, kEvLevel = 2, kEvDeath = 4, kEvWon = 8, kEvGameOver = 16, kEvStall = 32, kEvRollback = 64 };

static __device__ Upd reward_update(const Spec& G, const Sig& s, int frames, Tracker& e) {
    const bool has_p = e.has_prev != 0;
    Sig p;
    p.in_play = e.prev_in_play; p.progress_valid = e.prev_progress_valid; p.dying = e.prev_dying;
    p.has_lives = e.prev_has_lives; p.has_health = e.prev_has_health; p.has_score = e.prev_has_score;
    p.game_over = e.prev_game_over; p.won = e.prev_won; p.level = e.prev_level; p.lives = e.prev_lives;
    p.progress = e.prev_progress; p.health = e.prev_health; p.score = e.prev_score;
    e.has_prev = 1;
    e.prev_in_play = s.in_play; e.prev_progress_valid = s.progress_valid; e.prev_dying = s.dying;
    e.prev_has_lives = s.has_lives; e.prev_has_health = s.has_health; e.prev_has_score = s.has_score;
    e.prev_game_over = s.game_over; e.prev_won = s.won; e.prev_level = s.level; e.prev_lives = s.lives;
    e.prev_progress = s.progress; e.prev_health = s.health; e.prev_score = s.score;
    Upd out;
    out.reward = 0.0; out.done = true; out.events = 0; out.event_level = 0;
    for (int k = 0; k < kParts; ++k) out.part[k] = 0.0;
    if (e.done) return out;
    double r = 0.0, pt[kParts] = {0, 0, 0, 0, 0, 0, 0};
    u32 ev = 0;
    int ev_level = 0;
    bool fresh = false;
    if (s.in_play) {
        if (!e.has_best_level) {
            e.has_best_level = 1; e.best_level = s.level; e.has_best_progress = 0; e.score_used = 0.0;
        } else if (s.level > e.best_level + 1) {
            ev |= kEvSkip; ev_level = s.level; e.done = 1; e.end_reason = 3;
        } else if (s.level > e.best_level) {
            r = __dadd_rn(r, G.w_level); pt[1] = __dadd_rn(pt[1], G.w_level);
            ev |= kEvLevel; ev_level = s.level;
            e.best_level = s.level; e.has_best_progress = 0; e.score_used = 0.0;
            fresh = true;
        }
        if (s.level == e.best_level && s.progress_valid) {
            if (!e.has_best_progress) {
                e.has_best_progress = 1; e.best_progress = s.progress;
            } else if (s.progress > e.best_progress) {
                const double rp = __ddiv_rn(__dmul_rn(G.w_progress, __dsub_rn(s.progress, e.best_progress)), G.progress_unit);
                r = __dadd_rn(r, rp); pt[0] = __dadd_rn(pt[0], rp);
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
            r = __dadd_rn(r, G.w_death); pt[2] = __dadd_rn(pt[2], G.w_death);
            e.deaths += 1;
            ev |= kEvDeath;
            fresh = true;
        }
        if (s.in_play && p.in_play && s.has_health && p.has_health && s.health < p.health) {
            const double rd = __dmul_rn(G.w_damage, __dsub_rn(p.health, s.health));
            r = __dadd_rn(r, rd); pt[3] = __dadd_rn(pt[3], rd);
        }
        if (s.in_play && p.in_play && s.has_score && p.has_score && s.score > p.score) {
            double sr = __ddiv_rn(__dmul_rn(G.w_score, static_cast<double>(s.score - p.score)), G.score_unit);
            if (G.score_cap < sr) sr = G.score_cap;
            const double left = __dsub_rn(G.score_level_budget, e.score_used);
            if (left < sr) sr = left;
            if (sr > 0) { r = __dadd_rn(r, sr); pt[4] = __dadd_rn(pt[4], sr); e.score_used = __dadd_rn(e.score_used, sr); }
        }
    }
    if (has_p && !e.done && !death && !s.dying && !p.dying && !s.won && !s.game_over && s.in_play && p.in_play &&
        s.progress_valid && p.progress_valid && s.level == p.level && s.level == e.best_level &&
        __dsub_rn(p.progress, s.progress) >= __dmul_rn(G.rollback_drop, G.progress_unit)) {
        r = __dadd_rn(r, G.w_rollback); pt[6] = __dadd_rn(pt[6], G.w_rollback);
        ev |= kEvRollback;
    }
    if (!fresh && !e.done && has_p && s.in_play && p.in_play && s.progress_valid && p.progress_valid &&
        s.progress <= p.progress) {
        const double ci = __dmul_rn(G.idle_per_frame, static_cast<double>(frames));
        r = __dadd_rn(r, ci); pt[6] = __dadd_rn(pt[6], ci);
    }
    e.idle_frames = (fresh || !has_p) ? 0 : e.idle_frames + frames;
    if (s.won) {
        r = __dadd_rn(r, G.w_win); pt[5] = __dadd_rn(pt[5], G.w_win);
        ev |= kEvWon; e.done = 1; e.end_reason = 2;
    } else if (s.game_over) {
        ev |= kEvGameOver; e.done = 1; e.end_reason = 1;
    } else if (!e.done && G.stall_frames >= 0.0 && static_cast<double>(e.idle_frames) >= G.stall_frames) {
        r = __dadd_rn(r, G.w_stall); pt[6] = __dadd_rn(pt[6], G.w_stall);
        ev |= kEvStall; e.done = 1; e.end_reason = 4;
    }
    out.reward = r; out.done = e.done != 0; out.events = ev; out.event_level = ev_level;
    for (int k = 0; k < kParts; ++k) out.part[k] = pt[k];
    return out;
}

// ------------------------------------------------------------------------------------------------ env arrays

// A boot restart's outcome besides the machine record: the env's clock, fault code and tracker after the idle frames,
// the 4 neutral frames and the first tracker update.
struct RestartMeta {
    Tracker trk;
    u64 target;
    u32 ep_frame, fault;
    i32 ep_maxlvl;
    u32 ok;          // 1: template k was taken
};

struct GameArgs {   // one game slice
    CartView cart;
    Spec spec;
    u32 e0, n;                 // global env range
    const u8* recs;            // snapshot records: [1 + idle_tmpl][kRecBytes] (boot first)
    u32 idle_tmpl;
    u64 tmpl_target;
    u32 start_ok, select_ok;
    u32 game_e0;               // first env of the whole game (a range step moves e0, never this)
    // Level starts (rl/csrc/rlenv_core.cuh GameCtx lv_*): lv_cap saved states, slots < lv_levels level entrances,
    // the rest places. lv_deaths -1 = nothing saved; lv_claim = this decision's best arrival (deaths << 32 | env
    // within the game), ~0 = none. lv_cap 0 = level starts off.
    u32 lv_cap, lv_levels, lv_thresh, lv_weighted;
    u8* lv_rec;                // [lv_cap][kRecBytes]
    Tracker* lv_st;
    u64* lv_target;
    u32* lv_frame;
    i32* lv_deaths;
    unsigned long long* lv_claim;
    const u32* lv_cdf;         // [lv_cap] level pick CDF (lv_weighted)
    // Idle-frame chains of the saved slots: the state after k = 1..lv_idle_n idle frames (pad 0) from slot s, a pure
    // function of the slot (as the boot snapshot's idle records), made by k_chain when a slot's contents change.
    u32 lv_idle_n;             // idle_max
    u8* lv_idle_rec;           // [lv_cap][lv_idle_n][kRecBytes]
    u32* lv_idle_fault;        // [lv_cap][lv_idle_n] fault code after those frames
    u32* lv_chain_ok;          // [lv_cap] 1: the chain matches the slot
    StateView lv_scratch;      // emulation space of k_chain, env index = slot
    // Restart templates: a boot restart with k <= idle_tmpl idle frames (the boot snapshot's record k, then the 4
    // neutral frames with pad 0 and the first tracker update) is a pure function of k, so the whole outcome - machine
    // record, the 4 presentation slots, clock, fault, tracker and the first observation - is taken once from an env
    // that made it (k_tmpl_capture, after rlenv_start) and copied by k_restore instead of emulating and drawing it.
    u8* tm_rec;                // [idle_tmpl + 1][kRecBytes]
    u8* tm_nt;                 // [idle_tmpl + 1][4][2048] presentation slots
    u8* tm_oam;                // [idle_tmpl + 1][4][256]
    u8* tm_chr;                // [idle_tmpl + 1][4][8192] (CHR-RAM carts)
    u8* tm_bank;               // [idle_tmpl + 1][4]
    u8* tm_pix;                // [idle_tmpl + 1][4][224][240] colour numbers of the first observation
    u8* tm_emph;               // [idle_tmpl + 1][4][224]
    RestartMeta* tm_meta;      // [idle_tmpl + 1]
};

struct EnvArgs {
    StateView st;
    // per env (global index)
    Tracker* trk;
    Dropout* drop;
    u64* target;
    u32* ep_frame;
    int16_t* prev_applied;
    u64* sticky_seed;
    u64* sticky_ctr;
    u32* episode;
    float* ep_ret;
    i32* ep_len;
    i32* ep_maxlvl;
    i32* ep_idle;
    u32* fault;
    u8* resetting;
    u8* render_seq;     // [N, 4] frames left to the sequential renderer by the last render pass
    unsigned long long* render_stats;   // [2] frames drawn by the sequential renderer, split lines drawn by the walk
    u8* tm_used;        // [N] 1: the env's restart was copied from a restart template (no restart frames to run)
    double* ep_acc;     // optional [4]: finished episodes, their deaths, their returns, level events (added here)
    // restart list
    u32* list;
    u32* list_count;
    // caller buffers
    const int16_t* actions;
    u8* obs; u8* emph; float* reward; u8* done; u8* masks; u8* timeline; u8* pads; u32* events; float* info;
    float* parts;
    u8* packed;     // optional [N, 4, 224, 180] packed 6-bit pictures (replaces obs when set)
    i32* ep_start;      // [N] slot the episode started from, -1 = power-on; nullptr = level starts off
    u8* lv_chained;     // [N] 1: k_restore copied the level start's state after its idle frames (none left to run)
    i32* start_out;     // optional [N]: ep_start of the episode that just ended (where done)
    i32* level_out;     // optional [N]: level after the decision's update, -1 = not known yet
    float* progress_out;   // optional [N]: within-level progress / progress_unit, NaN = not valid now
    u64 run_seed;
    i32 sticky, idle_max, dropout, no_render, episode_level_end;
};

// ------------------------------------------------------------------------------------------------ records

// env slot <- record (whole console state; the record's frozen frame goes to presentation slot 0); threads tid of
// nt share the copy (one thread: 0 of 1)
static __device__ void scatter_record(const StateView& S, u32 e, const u8* rec, bool chr_ram, u32 tid = 0, u32 nt = 1) {
    const u32* rr = reinterpret_cast<const u32*>(rec + kRecRegs);
    for (u32 w = tid; w < static_cast<u32>(kRegWords); w += nt)
        S.regs[static_cast<u64>(w) * S.Np + e] = w == static_cast<u32>(R_FSLOT) ? 0u
                                                : w == static_cast<u32>(R_CHRD) ? 1u : rr[w];   // shared CHR stale
    const u32* ram = reinterpret_cast<const u32*>(rec + kRecRam);
    for (u32 i = tid; i < kRamWords; i += nt) S.ram[static_cast<u64>(i) * S.Np + e] = ram[i];
    const u32* pr = reinterpret_cast<const u32*>(rec + kRecPrgRam);
    for (u32 i = tid; i < kPrgRamWords; i += nt) S.prg_ram[static_cast<u64>(i) * S.Np + e] = pr[i];
    auto cp = [tid, nt](u8* d, const u8* s, u32 n) {
        uint4* dv = reinterpret_cast<uint4*>(d);
        const uint4* sv = reinterpret_cast<const uint4*>(s);
        for (u32 i = tid; i < n / 16; i += nt) dv[i] = sv[i];
    };
    cp(S.oam + static_cast<u64>(e) * kOamBytes, rec + kRecOam, kOamBytes);
    cp(S.nt + static_cast<u64>(e) * kNtBytes, rec + kRecNt, kNtBytes);
    cp(S.pal + static_cast<u64>(e) * kPalBytes, rec + kRecPal, kPalBytes);
    if (chr_ram) cp(S.chr_ram + static_cast<u64>(e) * kChrRamBytes, rec + kRecChrRam, kChrRamBytes);
    cp(reinterpret_cast<u8*>(S.log + static_cast<u64>(e) * kLogBanks * kLogBankWords), rec + kRecLog, kLogBanks * kLogBankWords * 4);
    const u64 sl = static_cast<u64>(e) * 4;
    cp(S.snap_nt + sl * kNtBytes, rec + kRecSnapNt, kNtBytes);
    cp(S.snap_oam + sl * kOamBytes, rec + kRecSnapOam, kOamBytes);
    if (chr_ram && S.snap_chr) cp(S.snap_chr + sl * kChrRamBytes, rec + kRecChrRam, kChrRamBytes);
    if (tid == 0) {
        S.slot_bank[sl] = static_cast<u8>((rr[R_PPU2] >> 8) & kLcBank);
        if (S.chr_ref) S.chr_ref[sl] = 0;
    }
}

// The snapshot record an episode restarts from: a saved level start, the boot snapshot after k idle frames, or the
// boot snapshot (rl/csrc/rlenv_core.cuh:236-243).
// A level start with idle frames takes its slot's idle chain record when the chain is made (`chained`).
__device__ __forceinline__ const u8* restart_record(const GameArgs& g, const EnvArgs& A, u32 ge, bool& chained) {
    const int lv = A.ep_start ? A.ep_start[ge] : -1;
    const int idle = A.ep_idle[ge];
    chained = false;
    if (lv >= 0) {
        if (idle > 0 && g.lv_idle_rec && static_cast<u32>(idle) <= g.lv_idle_n && g.lv_chain_ok[lv]) {
            chained = true;
            return g.lv_idle_rec + (static_cast<u64>(lv) * g.lv_idle_n + static_cast<u64>(idle - 1)) * kRecBytes;
        }
        return g.lv_rec + static_cast<u64>(lv) * kRecBytes;
    }
    const int k = idle <= static_cast<int>(g.idle_tmpl) ? idle : 0;
    return g.recs + static_cast<u64>(k) * kRecBytes;
}

// record <- env slot; threads tid of nt share the copy (one thread: 0 of 1)
static __device__ void gather_record(const StateView& S, u32 e, u8* rec, bool chr_ram, u32 tid = 0, u32 nt = 1) {
    u32* rr = reinterpret_cast<u32*>(rec + kRecRegs);
    for (u32 w = tid; w < 64; w += nt) rr[w] = w < static_cast<u32>(kRegWords) ? S.regs[static_cast<u64>(w) * S.Np + e] : 0u;
    u32* ram = reinterpret_cast<u32*>(rec + kRecRam);
    for (u32 i = tid; i < kRamWords; i += nt) ram[i] = S.ram[static_cast<u64>(i) * S.Np + e];
    u32* pr = reinterpret_cast<u32*>(rec + kRecPrgRam);
    for (u32 i = tid; i < kPrgRamWords; i += nt) pr[i] = S.prg_ram[static_cast<u64>(i) * S.Np + e];
    auto cp = [tid, nt](u8* d, const u8* s, u32 n) {
        uint4* dv = reinterpret_cast<uint4*>(d);
        const uint4* sv = reinterpret_cast<const uint4*>(s);
        for (u32 i = tid; i < n / 16; i += nt) dv[i] = sv[i];
    };
    cp(rec + kRecOam, S.oam + static_cast<u64>(e) * kOamBytes, kOamBytes);
    cp(rec + kRecNt, S.nt + static_cast<u64>(e) * kNtBytes, kNtBytes);
    cp(rec + kRecPal, S.pal + static_cast<u64>(e) * kPalBytes, kPalBytes);
    if (chr_ram) cp(rec + kRecChrRam, S.chr_ram + static_cast<u64>(e) * kChrRamBytes, kChrRamBytes);
    else for (u32 i = tid; i < kChrRamBytes / 4; i += nt) reinterpret_cast<u32*>(rec + kRecChrRam)[i] = 0;
    cp(rec + kRecLog, reinterpret_cast<const u8*>(S.log + static_cast<u64>(e) * kLogBanks * kLogBankWords), kLogBanks * kLogBankWords * 4);
    const u32 fs = S.regs[static_cast<u64>(R_FSLOT) * S.Np + e];
    const u64 sl = static_cast<u64>(e) * 4 + fs;
    cp(rec + kRecSnapNt, S.snap_nt + sl * kNtBytes, kNtBytes);
    cp(rec + kRecSnapOam, S.snap_oam + sl * kOamBytes, kOamBytes);
}

// ------------------------------------------------------------------------------------------------ phases

static __device__ void write_controls(const GameArgs& g, const EnvArgs& A, u32 ge) {
    const Dropout& d = A.drop[ge];
    const int dr = dropped_now(d);
    u32 dp = 0x1FF, ma = 7, mb = 7;
    const u32 ms = g.start_ok ? 3u : 1u, msel = g.select_ok ? 3u : 1u;
    if (dr >= 0 && dr < 4) for (u32 k = 0; k < 9; ++k) if (dpad_bits(k) & (0x10u << dr)) dp &= ~(1u << k);
    if (dr == 4) ma &= ~2u;
    if (dr == 6) ma &= ~4u;
    if (dr == 5) mb &= ~2u;
    if (dr == 7) mb &= ~4u;
    u8* mo = A.masks + static_cast<u64>(ge) * kMaskBytes;
    for (int i = 0; i < 9; ++i) mo[i] = (dp >> i) & 1u;
    for (int i = 0; i < 3; ++i) mo[9 + i] = (ma >> i) & 1u;
    for (int i = 0; i < 3; ++i) mo[12 + i] = (mb >> i) & 1u;
    for (int i = 0; i < 2; ++i) mo[15 + i] = (ms >> i) & 1u;
    for (int i = 0; i < 2; ++i) mo[17 + i] = (msel >> i) & 1u;
    // timeline [8, 45]: zeros, then a 1 where input b is off at decision now + j
    u8* tl = A.timeline + static_cast<u64>(ge) * kTimelineBytes;
    u32* tw = reinterpret_cast<u32*>(tl);   // 360 bytes per env: 4-byte aligned rows
    for (int i = 0; i < kTimelineBytes / 4; ++i) tw[i] = 0u;
    for (int j = 0; j < kTimeline; ++j) {
        const int b = d.ring[(d.head + j) % kRing];
        if (b >= 0) tl[b * kTimeline + j] = 1;
    }
}

// rl/csrc/rlenv_core.cuh:208-263: idle count, level-start coin and pick (drawn only when level starts are on), and
// the episode's scalars from the chosen snapshot; the snapshot record itself is copied into the env by k_restore.
static __device__ void reset_state(const GameArgs& g, const EnvArgs& A, u32 ge) {
    const u32 ep = ++A.episode[ge];
    const u64 seed = splitmix64(splitmix64(A.run_seed ^ 0xD20F0D20F0ull) ^ (static_cast<u64>(ge) << 40) ^ static_cast<u64>(ep));
    const u64 ss = splitmix64(seed ^ 0x5717C4A55EEDull);
    u64 ctr = 0;
    int idle = 0;
    if (A.idle_max > 0) idle = static_cast<int>(rand_below(ss, ctr, static_cast<u32>(A.idle_max + 1)));
    int lv = -1;
    if (g.lv_cap > 0 && g.lv_thresh != 0 && rand_u32(ss, ctr) < g.lv_thresh) {
        u32 saved = 0;
        for (u32 s = 0; s < g.lv_cap; ++s) saved += g.lv_deaths[s] >= 0 ? 1u : 0u;
        if (g.lv_weighted) {
            const u32 u = rand_u32(ss, ctr);
            for (u32 s = 0; s < g.lv_cap && lv < 0; ++s)
                if (u < g.lv_cdf[s]) lv = static_cast<int>(s);
        } else if (saved > 0) {
            u32 pick = rand_below(ss, ctr, saved);
            for (u32 s = 0; s < g.lv_cap && lv < 0; ++s)
                if (g.lv_deaths[s] >= 0 && pick-- == 0) lv = static_cast<int>(s);
        }
    }
    A.sticky_seed[ge] = ss;
    A.sticky_ctr[ge] = ctr;
    const int k = lv < 0 && idle <= static_cast<int>(g.idle_tmpl) ? idle : 0;
    if (lv >= 0) {
        A.target[ge] = g.lv_target[lv];
        A.ep_frame[ge] = g.lv_frame[lv];
        A.trk[ge] = g.lv_st[lv];
    } else {
        A.target[ge] = g.tmpl_target + static_cast<u64>(k) * kFrameDots;
        A.ep_frame[ge] = static_cast<u32>(k);
        Tracker t;
        memset(&t, 0, sizeof t);
        A.trk[ge] = t;
    }
    if (A.ep_start) A.ep_start[ge] = lv;
    A.fault[ge] = 0;
    Dropout d;
    dropout_reset(d, seed, A.dropout != 0);
    A.drop[ge] = d;
    A.prev_applied[ge] = 0;
    A.ep_idle[ge] = idle;
    A.resetting[ge] = 1;
}

// ------------------------------------------------------------------------------------------------ kernels

// Emulation: kFramesWarps warps per block, kEnvsPerWarp envs per warp, consoles staged in shared memory for the whole
// launch.
// `restart` = 0: the 4 frames of a decision for envs [e0, e0+n); 1: restart frames for the listed envs.
// Shared memory of an emulation block: kFramesWarps console stagings, the decode table, the cart's PRG window.
constexpr std::size_t kDtabOff = kFramesWarps * sizeof(EmuShared);
constexpr std::size_t kFramesSmem = kDtabOff + 256 * sizeof(u32);   // + the cart's staged PRG window
// static: the board units may compile different shapes (GR_ENVS_PER_WARP / GR_FRAMES_WARPS), each its own copy
static inline std::size_t frames_smem(const CartView& c) { return kFramesSmem + c.prg_stage_bytes; }
static inline u32 frames_blocks(u32 n) { return (n + kEnvsPerWarp * kFramesWarps - 1) / (kEnvsPerWarp * kFramesWarps); }

// The cart's PRG window into shared memory (threads tid of nthreads, 16-byte vectors).
__device__ __forceinline__ void stage_prg(const CartView& c, u8* dst, u32 tid, u32 nthreads) {
    const uint4* src = reinterpret_cast<const uint4*>(c.prg + c.prg_stage_base);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (u32 i = tid; i < c.prg_stage_bytes / 16; i += nthreads) d[i] = __ldg(src + i);
}

template <u32 BOARD>
__global__ void __launch_bounds__(32 * kFramesWarps, 1) k_frames(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A, int restart) {
    extern __shared__ __align__(16) u8 smem_raw[];
    const u32 lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    EmuShared& sh = reinterpret_cast<EmuShared*>(smem_raw)[wid];
    u32* dtab = reinterpret_cast<u32*>(smem_raw + kDtabOff);
    u8* prg_s = smem_raw + kFramesSmem;
    for (u32 i = threadIdx.x; i < 256; i += blockDim.x) dtab[i] = kDecode.t[i];
    stage_prg(g.cart, prg_s, threadIdx.x, blockDim.x);
    __syncthreads();
    const u32 total = restart ? *A.list_count : g.n;
    // each warp its own run of kEnvsPerWarp envs; no block-wide synchronisation from here on
    for (u32 base = (blockIdx.x * kFramesWarps + wid) * kEnvsPerWarp; base < total;
         base += gridDim.x * kFramesWarps * kEnvsPerWarp) {
        const u32 k = base + lane;
        u32 ge = 0;
        bool valid = lane < kEnvsPerWarp && k < total;
        if (valid) {
            ge = restart ? A.list[k] : g.e0 + k;
            valid = ge >= g.e0 && ge < g.e0 + g.n && !(restart && A.tm_used[ge]);
        }
        Emu<BOARD> m(A.st, g.cart, valid ? ge : g.e0, lane, sh, dtab, prg_s);
        m.froze = 0;
        if (valid) { m.stage_in(); m.load(); }
        m.refresh_shared_chr(valid);
        u32 fault = valid ? A.fault[ge] : 0u;
        u64 target = valid ? A.target[ge] : 0ull;
        u32 ep_frame = valid ? A.ep_frame[ge] : 0u;
        // per lane: frames to run (decision: 4; restart: idle frames beyond the copied snapshot, then 4 neutral
        // frames, rl/csrc/rlenv_core.cuh:311-328) - one step_until call site for the whole warp
        int dr = -1, prev = 0, act = 0, extra = 0;
        u64 sctr = 0, sseed = 0;
        if (valid) {
            if (!restart) {
                dr = dropped_now(A.drop[ge]);
                sctr = A.sticky_ctr[ge];
                sseed = A.sticky_seed[ge];
                prev = A.prev_applied[ge];
                act = A.actions[ge];
            } else {
                const int idle = A.ep_idle[ge];
                // a level start emulates every idle frame unless its slot's chain supplied them
                const bool lv = A.ep_start && A.ep_start[ge] >= 0;
                const bool chained = lv && A.lv_chained && A.lv_chained[ge];
                extra = lv ? (chained ? 0 : idle) : (idle <= static_cast<int>(g.idle_tmpl) ? 0 : idle);
            }
        }
        const int nfr = extra + kFramesPerDecision;
        const int most = __reduce_max_sync(0xFFFFFFFFu, valid ? nfr : 0);
        u32 pads4 = 0;
        for (int i = 0; i < most; ++i) {
            const bool mine = valid && i < nfr;
            if (mine) {
                u32 pad = 0;
                if (!restart) {
                    Move mv = unpack_move(act);
                    if (A.sticky && rand_u32(sseed, sctr) < kSticky32)
                        mv = restrict_move(unpack_move(prev), dr, g.start_ok != 0, g.select_ok != 0);
                    prev = pack_move(mv);
                    pad = pad_byte(mv, ep_frame);
                    pads4 |= pad << (8 * i);
                }
                m.pad = pad;
                m.slot = i < extra ? 0u : static_cast<u32>(i - extra);
            }
            const u32 fl = m.step_until(target, mine && fault == 0);
            m.snapshot_frozen();
            if (mine) {
                if (fl) fault = fl;
                m.finish_slot();
                target += kFrameDots;
                ep_frame += 1;
            }
        }
        if (valid && !restart) {
            A.sticky_ctr[ge] = sctr;
            A.prev_applied[ge] = static_cast<int16_t>(prev);
            reinterpret_cast<u32*>(A.pads)[ge] = pads4;
        }
        if (valid) {
            m.store();
            m.stage_out();
            A.fault[ge] = fault;
            A.target[ge] = target;
            A.ep_frame[ge] = ep_frame;
        }
        if (restart && valid) {
            // ph_reset_finish_controls: first tracker update (no reward), counters, controls
            Tracker t = A.trk[ge];
            (void)reward_update(g.spec, observe_synth(A.st, ge), A.ep_idle[ge] + kFramesPerDecision, t);
            A.trk[ge] = t;
            A.ep_ret[ge] = 0.0f;
            A.ep_len[ge] = 0;
            const int sl = A.ep_start ? A.ep_start[ge] : -1;   // a place: its level is the tracker's
            A.ep_maxlvl[ge] = sl >= static_cast<int>(g.lv_levels) ? (t.has_best_level ? t.best_level : 0) : sl > 0 ? sl : 0;
            A.resetting[ge] = 0;
            write_controls(g, A, ge);
        }
        __syncwarp();
    }
}

// After a decision's frames: reward, outputs, episode end (rl/csrc/rlenv_core.cuh:266-309).
static __global__ void __launch_bounds__(128) k_finish(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A, int start) {
    const u32 k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= g.n) return;
    const u32 ge = g.e0 + k;
    bool done;
    if (start) {
        done = true;
    } else {
        Tracker t = A.trk[ge];
        const Upd u = reward_update(g.spec, observe_synth(A.st, ge), kFramesPerDecision, t);
        A.trk[ge] = t;
        const bool faulted = A.fault[ge] != 0;
        const bool level_clear = !u.done && !faulted && A.episode_level_end >= 0 && (u.events & kEvLevel) &&
                                 u.event_level == A.episode_level_end + 1;
        const bool frame_limit = !u.done && !faulted && !level_clear && g.spec.frame_limit > 0.0 &&
                                 static_cast<double>(A.ep_frame[ge]) >= g.spec.frame_limit;
        done = u.done || faulted || level_clear || frame_limit;
        const float r = faulted ? 0.0f : __double2float_rn(u.reward);
        A.reward[ge] = r;
        if (A.parts)
            for (int q = 0; q < kParts; ++q) A.parts[static_cast<u64>(ge) * kParts + q] = faulted ? 0.0f : __double2float_rn(u.part[q]);
        A.done[ge] = done ? 1 : 0;
        A.events[ge] = u.events;
        const float ret = __fadd_rn(A.ep_ret[ge], r);
        A.ep_ret[ge] = ret;
        const i32 len = A.ep_len[ge] + 1;
        A.ep_len[ge] = len;
        if (u.event_level > A.ep_maxlvl[ge]) A.ep_maxlvl[ge] = u.event_level;
        Dropout d = A.drop[ge];
        dropout_advance(d, A.dropout != 0);
        A.drop[ge] = d;
        if (g.lv_cap > 0 && !done && (u.events & kEvLevel) && u.event_level >= 0 && u.event_level < static_cast<int>(g.lv_levels)) {
            const u64 dd = t.deaths < 0 ? 0u : static_cast<u64>(t.deaths);
            atomicMin(&g.lv_claim[u.event_level], static_cast<unsigned long long>((dd << 32) | (ge - g.game_e0)));
        }
        if (A.level_out) A.level_out[ge] = t.has_best_level ? t.best_level : -1;
        if (A.progress_out)
            A.progress_out[ge] = t.has_prev && t.prev_progress_valid
                ? __double2float_rn(__ddiv_rn(t.prev_progress, g.spec.progress_unit)) : __int_as_float(0x7FC00000);
        if (done) {
            if (A.start_out) A.start_out[ge] = A.ep_start ? A.ep_start[ge] : -1;
            float* inf = A.info + static_cast<u64>(ge) * kInfo;
            inf[0] = ret;
            inf[1] = static_cast<float>(len);
            inf[2] = static_cast<float>(faulted ? 5 : level_clear ? 6 : frame_limit ? 7 : t.end_reason);
            inf[3] = static_cast<float>(t.deaths);
            inf[4] = static_cast<float>(A.ep_maxlvl[ge]);
            inf[5] = t.overflow ? 1.0f : 0.0f;
            inf[6] = static_cast<float>(A.ep_idle[ge]);
            inf[7] = static_cast<float>(A.episode[ge]);
        }
        if (A.ep_acc) {   // the rollout's episode counters: one fp64 atomic per finished episode or level event
            if (done) {
                atomicAdd(&A.ep_acc[0], 1.0);
                atomicAdd(&A.ep_acc[1], static_cast<double>(t.deaths));
                atomicAdd(&A.ep_acc[2], static_cast<double>(ret));
            }
            if (u.events & kEvLevel) atomicAdd(&A.ep_acc[3], 1.0);
        }
    }
    if (done) {
        reset_state(g, A, ge);
        const u32 slot = atomicAdd(A.list_count, 1u);
        A.list[slot] = ge;
    } else {
        write_controls(g, A, ge);
    }
}

// A boot restart with k idle frames that has a template (0 <= k <= idle_tmpl, template taken).
__device__ __forceinline__ bool tmpl_restart(const GameArgs& g, const EnvArgs& A, u32 ge, int& k) {
    k = A.ep_idle[ge];
    if (!g.tm_meta || (A.ep_start && A.ep_start[ge] >= 0)) return false;
    return k >= 0 && k <= static_cast<int>(g.idle_tmpl) && g.tm_meta[k].ok != 0u;
}

// Restarting envs <- their snapshot records (after k_finish listed them): one block per listed env. A boot restart
// with a template takes the template's whole outcome instead (record, presentation slots, first observation, clock,
// fault, tracker; controls from its own dropout state) and is left out of the restart frames and drawing.
static __global__ void __launch_bounds__(128) k_restore(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A) {
    const u32 total = *A.list_count;
    const bool chr_ram = g.cart.chr == nullptr;
    for (u32 k = blockIdx.x; k < total; k += gridDim.x) {
        const u32 ge = A.list[k];
        int tk;
        if (tmpl_restart(g, A, ge, tk)) {
            const u64 t4 = static_cast<u64>(tk) * 4;
            scatter_record(A.st, ge, g.tm_rec + static_cast<u64>(tk) * kRecBytes, chr_ram, threadIdx.x, blockDim.x);
            const u64 s4 = static_cast<u64>(ge) * 4;
            {   // presentation slots
                const uint4* src = reinterpret_cast<const uint4*>(g.tm_nt + t4 * kNtBytes);
                uint4* dst = reinterpret_cast<uint4*>(A.st.snap_nt + s4 * kNtBytes);
                for (u32 i = threadIdx.x; i < 4 * kNtBytes / 16; i += blockDim.x) dst[i] = src[i];
                const uint4* so = reinterpret_cast<const uint4*>(g.tm_oam + t4 * kOamBytes);
                uint4* doam = reinterpret_cast<uint4*>(A.st.snap_oam + s4 * kOamBytes);
                for (u32 i = threadIdx.x; i < 4 * kOamBytes / 16; i += blockDim.x) doam[i] = so[i];
                if (chr_ram && A.st.snap_chr) {
                    const uint4* sc = reinterpret_cast<const uint4*>(g.tm_chr + t4 * kChrRamBytes);
                    uint4* dc = reinterpret_cast<uint4*>(A.st.snap_chr + s4 * kChrRamBytes);
                    for (u32 i = threadIdx.x; i < 4 * kChrRamBytes / 16; i += blockDim.x) dc[i] = sc[i];
                }
                if (threadIdx.x < 4) {
                    A.st.slot_bank[s4 + threadIdx.x] = g.tm_bank[t4 + threadIdx.x];
                    if (A.st.chr_ref) A.st.chr_ref[s4 + threadIdx.x] = 0;   // the template's copies are the slots' own
                }
            }
            if (!A.no_render) {   // the first observation: colour numbers, or 6-bit packed (4 pixels -> 3 bytes)
                const u32* px = reinterpret_cast<const u32*>(g.tm_pix + t4 * kObsPixels);
                if (A.packed) {
                    u8* dst = A.packed + s4 * (kObsPixels / 4 * 3);
                    for (u32 i = threadIdx.x; i < 4 * kObsPixels / 4; i += blockDim.x) {
                        const u32 w = px[i];
                        const u32 v = (w & 0x3Fu) | (((w >> 8) & 0x3Fu) << 6) | (((w >> 16) & 0x3Fu) << 12) | (((w >> 24) & 0x3Fu) << 18);
                        dst[3 * i] = static_cast<u8>(v); dst[3 * i + 1] = static_cast<u8>(v >> 8); dst[3 * i + 2] = static_cast<u8>(v >> 16);
                    }
                } else {
                    const uint4* src = reinterpret_cast<const uint4*>(px);
                    uint4* dst = reinterpret_cast<uint4*>(A.obs + s4 * kObsPixels);
                    for (u32 i = threadIdx.x; i < 4 * kObsPixels / 16; i += blockDim.x) dst[i] = src[i];
                }
                const u8* se = g.tm_emph + t4 * kObsH;
                u8* de = A.emph + s4 * kObsH;
                for (u32 i = threadIdx.x; i < 4 * kObsH; i += blockDim.x) de[i] = se[i];
            }
            __syncthreads();
            if (threadIdx.x == 0) {   // ph_reset_finish_controls as the template made it, then this env's controls
                const RestartMeta& M = g.tm_meta[tk];
                A.trk[ge] = M.trk;
                A.target[ge] = M.target;
                A.ep_frame[ge] = M.ep_frame;
                A.fault[ge] = M.fault;
                A.ep_ret[ge] = 0.0f;
                A.ep_len[ge] = 0;
                A.ep_maxlvl[ge] = M.ep_maxlvl;
                A.resetting[ge] = 0;
                A.tm_used[ge] = 1;
                if (A.lv_chained) A.lv_chained[ge] = 0;
                write_controls(g, A, ge);
            }
            __syncthreads();
            continue;
        }
        bool chained;
        const u8* rec = restart_record(g, A, ge, chained);
        scatter_record(A.st, ge, rec, chr_ram, threadIdx.x, blockDim.x);
        if (threadIdx.x == 0) {
            A.tm_used[ge] = 0;
            if (A.lv_chained) {
                A.lv_chained[ge] = chained ? 1 : 0;
                if (chained) {   // the idle frames are in the record: the episode's clock and fault move on with them
                    const int lv = A.ep_start[ge], idle = A.ep_idle[ge];
                    A.target[ge] += static_cast<u64>(idle) * kFrameDots;
                    A.ep_frame[ge] += static_cast<u32>(idle);
                    A.fault[ge] = g.lv_idle_fault[static_cast<u64>(lv) * g.lv_idle_n + static_cast<u64>(idle - 1)];
                }
            }
        }
        __syncthreads();
    }
}

// Restart templates from the envs that just started (after rlenv_start, pictures drawn): block k takes the lowest env
// of the game slice whose first episode began from the boot snapshot with k idle frames; none: template k stays off.
static __global__ void __launch_bounds__(128) k_tmpl_capture(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A) {
    const u32 tk = blockIdx.x;
    __shared__ u32 best;
    if (threadIdx.x == 0) best = 0xFFFFFFFFu;
    __syncthreads();
    for (u32 i = threadIdx.x; i < g.n; i += blockDim.x) {
        const u32 ge = g.e0 + i;
        if (A.ep_idle[ge] == static_cast<int>(tk) && !(A.ep_start && A.ep_start[ge] >= 0) && A.resetting[ge] == 0) {
            atomicMin(&best, ge);
            break;
        }
    }
    __syncthreads();
    const u32 ge = best;
    RestartMeta& M = g.tm_meta[tk];
    if (ge == 0xFFFFFFFFu) {
        if (threadIdx.x == 0) M.ok = 0;
        return;
    }
    const bool chr_ram = g.cart.chr == nullptr;
    const u64 t4 = static_cast<u64>(tk) * 4, s4 = static_cast<u64>(ge) * 4;
    gather_record(A.st, ge, g.tm_rec + static_cast<u64>(tk) * kRecBytes, chr_ram, threadIdx.x, blockDim.x);
    {
        const uint4* src = reinterpret_cast<const uint4*>(A.st.snap_nt + s4 * kNtBytes);
        uint4* dst = reinterpret_cast<uint4*>(g.tm_nt + t4 * kNtBytes);
        for (u32 i = threadIdx.x; i < 4 * kNtBytes / 16; i += blockDim.x) dst[i] = src[i];
        const uint4* so = reinterpret_cast<const uint4*>(A.st.snap_oam + s4 * kOamBytes);
        uint4* doam = reinterpret_cast<uint4*>(g.tm_oam + t4 * kOamBytes);
        for (u32 i = threadIdx.x; i < 4 * kOamBytes / 16; i += blockDim.x) doam[i] = so[i];
        if (chr_ram && A.st.snap_chr) {   // each slot's CHR as drawn (its own copy or the env's shared one)
            for (u32 f = 0; f < 4; ++f) {
                const bool shared = A.st.chr_ref && A.st.chr_ref[s4 + f];
                const uint4* sc = reinterpret_cast<const uint4*>(
                    shared ? A.st.chr_shared + static_cast<u64>(ge) * kChrRamBytes : A.st.snap_chr + (s4 + f) * kChrRamBytes);
                uint4* dc = reinterpret_cast<uint4*>(g.tm_chr + (t4 + f) * kChrRamBytes);
                for (u32 i = threadIdx.x; i < kChrRamBytes / 16; i += blockDim.x) dc[i] = sc[i];
            }
        }
        if (threadIdx.x < 4) g.tm_bank[t4 + threadIdx.x] = A.st.slot_bank[s4 + threadIdx.x];
    }
    u32* px = reinterpret_cast<u32*>(g.tm_pix + t4 * kObsPixels);
    if (A.packed) {   // 3 bytes -> 4 colour numbers
        const u8* src = A.packed + s4 * (kObsPixels / 4 * 3);
        for (u32 i = threadIdx.x; i < 4 * kObsPixels / 4; i += blockDim.x) {
            const u32 v = src[3 * i] | (static_cast<u32>(src[3 * i + 1]) << 8) | (static_cast<u32>(src[3 * i + 2]) << 16);
            px[i] = (v & 0x3Fu) | (((v >> 6) & 0x3Fu) << 8) | (((v >> 12) & 0x3Fu) << 16) | (((v >> 18) & 0x3Fu) << 24);
        }
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(A.obs + s4 * kObsPixels);
        for (u32 i = threadIdx.x; i < 4 * kObsPixels / 16; i += blockDim.x) reinterpret_cast<uint4*>(px)[i] = src[i];
    }
    for (u32 i = threadIdx.x; i < 4 * kObsH; i += blockDim.x) g.tm_emph[t4 * kObsH + i] = A.emph[s4 * kObsH + i];
    __syncthreads();
    if (threadIdx.x == 0) {
        M.trk = A.trk[ge];
        M.target = A.target[ge];
        M.ep_frame = A.ep_frame[ge];
        M.fault = A.fault[ge];
        M.ep_maxlvl = A.ep_maxlvl[ge];
        M.ok = 1;
    }
}

// Level-start saves after a decision's k_finish (rl/csrc/rlenv.cu:89-97, rl/csrc/rlenv_core.cuh:344-387): block s
// takes slot s's claimed arrival when nothing is saved yet or it died no more often; the block copies the env's
// state record, then thread 0 commits the tracker, frame target and deaths and clears the claim.
static __global__ void __launch_bounds__(128) k_archive(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A) {
    const u32 s = blockIdx.x;
    const unsigned long long cl = g.lv_claim[s];
    if (cl == ~0ull) return;   // same for the whole block
    const bool take = g.lv_deaths[s] < 0 || static_cast<i32>(cl >> 32) <= g.lv_deaths[s];
    const u32 ge = g.game_e0 + static_cast<u32>(cl & 0xFFFFFFFFull);
    if (take) gather_record(A.st, ge, g.lv_rec + static_cast<u64>(s) * kRecBytes, g.cart.chr == nullptr, threadIdx.x, blockDim.x);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (take) {
            g.lv_st[s] = A.trk[ge];
            g.lv_target[s] = A.target[ge];
            g.lv_frame[s] = A.ep_frame[ge];
            g.lv_deaths[s] = static_cast<i32>(cl >> 32);
            if (g.lv_chain_ok) g.lv_chain_ok[s] = 0;   // new contents: the next decision's k_chain remakes the chain
        }
        g.lv_claim[s] = ~0ull;
    }
}

// Place saves (rl/places.py; rl/csrc/rlenv.cu:99-107): block j copies env env_idx[j] of the game (index within the
// game) into slot slot_idx[j], skipped unless lv_levels <= slot < lv_cap; the no-progress clock restarts.
static __global__ void __launch_bounds__(128) k_place_save(const __grid_constant__ GameArgs g, const __grid_constant__ EnvArgs A,
                                                           const i32* env_idx, const i32* slot_idx) {
    const i32 s = slot_idx[blockIdx.x], e = env_idx[blockIdx.x];
    if (s < static_cast<i32>(g.lv_levels) || s >= static_cast<i32>(g.lv_cap) || e < 0 || e >= static_cast<i32>(g.n)) return;
    const u32 ge = g.game_e0 + static_cast<u32>(e);
    gather_record(A.st, ge, g.lv_rec + static_cast<u64>(s) * kRecBytes, g.cart.chr == nullptr, threadIdx.x, blockDim.x);
    __syncthreads();
    if (threadIdx.x == 0) {
        Tracker t = A.trk[ge];
        t.idle_frames = 0;
        g.lv_st[s] = t;
        g.lv_target[s] = A.target[ge];
        g.lv_frame[s] = A.ep_frame[ge];
        g.lv_deaths[s] = 0;
        if (g.lv_chain_ok) g.lv_chain_ok[s] = 0;
    }
}

// Warp per (env, frame) of this game slice (or of the restart list), grid-stride: the warp walks the frame's log
// (phase 1) and draws it from the walk (phase 2); a frame with a write inside a line's drawn part is flagged for
// k_render_seq instead. The sequential renderer lives in its own kernel, so this one needs 96 registers instead
// of 124; a frame per warp lets a short restart list spread over 4x as many warps.
struct RenderWarp {
    RWarp w;
    FrameWalk fw;
};
constexpr u32 kRenderWarps = 8;
static_assert((kRenderWarps & (kRenderWarps - 1u)) == 0u, "k_render_seq's item scan takes kRenderWarps as a power of two");
// Render blocks per SM the register budget is fitted to: 3 for the CHR-ROM boards whose draw path is lightest
// (NROM, UxROM: <= 85 registers), 2 for the others (up to 128 registers)
template <u32 BOARD> constexpr int render_min_blocks() { return (BOARD == kNrom || BOARD == kUxrom) ? 3 : 2; }
inline std::size_t render_smem(bool chrx_smem) {
    return 1024 + (chrx_smem ? 16384 : 0) + kRenderWarps * sizeof(RenderWarp);
}
inline std::size_t render_seq_smem(bool chrx_smem) {
    return 1024 + (chrx_smem ? 16384 : 0) + kRenderWarps * sizeof(RWarp);
}

// Item k of a render launch: env item k / frames, frame k % frames; false when the env is not drawn by this pass.
__device__ __forceinline__ bool render_item(const RenderArgs& R, u32 k, u32& ge, u32& f) {
    const u32 ei = k / R.frames;
    f = k - ei * R.frames;
    ge = R.list ? R.list[ei] : R.e0 + ei;
    if (R.list && (ge < R.e0 || ge >= R.e0 + R.count)) return false;
    if (R.skip && R.skip[ge]) return false;   // restarting: the restart pass draws its new episode's first frames
    return true;
}

template <u32 BOARD>
__device__ __forceinline__ void render_setup(const RenderArgs& R, u8* smem, u32*& spread, u32*& chrx) {
    spread = reinterpret_cast<u32*>(smem);                 // 1 KB
    chrx = spread + 256;                                   // 16 KB when staged
    for (u32 i = threadIdx.x; i < 256; i += blockDim.x) spread[i] = spread8(i);
    if (R.chrx_smem) for (u32 i = threadIdx.x; i < 4096; i += blockDim.x) chrx[i] = R.cart.chrx[i];
    __syncthreads();
}

template <u32 BOARD>
__global__ void __launch_bounds__(32 * kRenderWarps, render_min_blocks<BOARD>()) k_render(const __grid_constant__ RenderArgs R) {
    extern __shared__ __align__(16) u8 smem[];
    u32 *spread, *chrx;
    render_setup<BOARD>(R, smem, spread, chrx);
    RenderWarp* warps = reinterpret_cast<RenderWarp*>(smem + 1024 + (R.chrx_smem ? 16384 : 0));
    const u32 lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    RenderWarp& RW = warps[wid];
    Renderer<BOARD> rd(R, lane, R.chrx_smem ? chrx : R.cart.chrx, spread, RW.w);
    const u32 items = (R.list ? *R.list_count : R.count) * R.frames;
    for (u32 k = blockIdx.x * kRenderWarps + wid; k < items; k += gridDim.x * kRenderWarps) {
        u32 ge, f;
        if (!render_item(R, k, ge, f)) continue;
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        if constexpr (BOARD == kMmc2) {   // the latches move with the fetches: the sequential renderer draws it all
            if (lane == 0) R.seqf[sl] = 1u;
        } else if constexpr (Renderer<BOARD>::kSplitLines) {   // the walk draws the lines with mid-line writes itself
            u8* out = R.packed ? R.packed + sl * (kObsPixels / 4 * 3) : R.obs + sl * kObsPixels;
            rd.walk_frame(ge, f, RW.fw, out, R.packed != nullptr);
            if (lane == 0) R.seqf[sl] = RW.fw.seq ? 1u : 0u;
            if (!RW.fw.seq) rd.draw_fast(ge, f, RW.fw, out, R.emph + sl * kObsH, R.packed != nullptr);
        } else {
            rd.walk_frame(ge, f, RW.fw, nullptr, false);
            if (lane == 0) R.seqf[sl] = RW.fw.seq ? 1u : 0u;
            if (!RW.fw.seq) {
                u8* out = R.packed ? R.packed + sl * (kObsPixels / 4 * 3) : R.obs + sl * kObsPixels;
                rd.draw_fast(ge, f, RW.fw, out, R.emph + sl * kObsH, R.packed != nullptr);
            }
        }
        __syncwarp();
    }
}

// The frames k_render flagged (same launch arguments, after it on the same stream): the sequential renderer.
template <u32 BOARD>
__global__ void __launch_bounds__(32 * kRenderWarps, 2) k_render_seq(const __grid_constant__ RenderArgs R) {
    extern __shared__ __align__(16) u8 smem[];
    {   // most launches find no flagged frame: the block's items are scanned by all its threads first, and a block
        // with none returns before staging its tables (the same items as the warp loop below, 32 per warp at once)
        const u32 items = (R.list ? *R.list_count : R.count) * R.frames;
        const u32 step = gridDim.x * kRenderWarps;
        bool found = false;
        for (u32 k = blockIdx.x * kRenderWarps + (threadIdx.x & (kRenderWarps - 1u)) + (threadIdx.x / kRenderWarps) * step;
             k < items; k += 32u * step) {
            u32 ge, f;
            if (render_item(R, k, ge, f) && R.seqf[static_cast<u64>(ge) * 4 + f]) found = true;
        }
        if (!__syncthreads_or(found)) return;
    }
    u32 *spread, *chrx;
    render_setup<BOARD>(R, smem, spread, chrx);
    RWarp* warps = reinterpret_cast<RWarp*>(smem + 1024 + (R.chrx_smem ? 16384 : 0));
    const u32 lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    Renderer<BOARD> rd(R, lane, R.chrx_smem ? chrx : R.cart.chrx, spread, warps[wid]);
    const u32 items = (R.list ? *R.list_count : R.count) * R.frames;
    for (u32 k = blockIdx.x * kRenderWarps + wid; k < items; k += gridDim.x * kRenderWarps) {
        u32 ge, f;
        if (!render_item(R, k, ge, f)) continue;
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        if (!R.seqf[sl]) continue;
        u8* out = R.packed ? R.packed + sl * (kObsPixels / 4 * 3) : R.obs + sl * kObsPixels;
        rd.draw(ge, f, out, R.emph + sl * kObsH, R.packed != nullptr);
        if (lane == 0) atomicAdd(R.stats, 1ull);
        __syncwarp();
    }
}

// Idle-frame chains of the saved slots whose contents changed (block s = slot s, lane 0 emulates in the scratch
// space): the state after each of idle_max idle frames (pad 0, the reference's ph_reset_idle frames,
// rl/csrc/rlenv_core.cuh:311-317) from the slot, with the fault code so far. Runs before k_restore; a restart whose
// slot has its chain copies the record after its idle count instead of emulating the frames.
template <u32 BOARD>
__global__ void __launch_bounds__(32, 1) k_chain(const __grid_constant__ GameArgs g) {
    const u32 s = blockIdx.x;
    if (g.lv_chain_ok[s] || g.lv_deaths[s] < 0 || g.lv_idle_n == 0) return;   // same for the whole block
    extern __shared__ __align__(16) u8 smem_raw[];
    EmuShared& sh = *reinterpret_cast<EmuShared*>(smem_raw);
    u32* dtab = reinterpret_cast<u32*>(smem_raw + kDtabOff);
    u8* prg_s = smem_raw + kFramesSmem;
    const u32 lane = threadIdx.x;
    for (int i = lane; i < 256; i += 32) dtab[i] = kDecode.t[i];
    stage_prg(g.cart, prg_s, lane, 32);
    const StateView& S = g.lv_scratch;
    scatter_record(S, s, g.lv_rec + static_cast<u64>(s) * kRecBytes, g.cart.chr == nullptr, lane, 32);
    __syncwarp();
    const bool me = lane == 0;
    Emu<BOARD> m(S, g.cart, s, lane, sh, dtab, prg_s);
    m.froze = 0;
    if (me) { m.stage_in(); m.load(); }
    u64 target = g.lv_target[s];
    u32 fault = 0;
    for (u32 k = 0; k < g.lv_idle_n; ++k) {
        if (me) { m.pad = 0; m.slot = 0; }
        const u32 f = m.step_until(target, me && fault == 0);
        m.snapshot_frozen();
        if (me) {
            m.finish_slot();
            if (f && !fault) fault = f;
            target += kFrameDots;
            m.store();
            m.stage_out();
        }
        __syncwarp();
        gather_record(S, s, g.lv_idle_rec + (static_cast<u64>(s) * g.lv_idle_n + k) * kRecBytes, g.cart.chr == nullptr, lane, 32);
        if (me) g.lv_idle_fault[static_cast<u64>(s) * g.lv_idle_n + k] = fault;
        __syncwarp();
    }
    if (me) {
        __threadfence();
        g.lv_chain_ok[s] = 1;
    }
}

// ------------------------------------------------------------------------------------------------ set-up kernels

// Power-on of env slot `e` (NeSLE cold reset, restated; RAM 0xFF as rl/csrc/rlenv_build.hpp:86), then the boot:
// `boot_n` frames with the given pads; after the boot and after each of `idle_n` further idle frames the state is
// written as a snapshot record. One warp, lane 0 emulates.
template <u32 BOARD>
__global__ void __launch_bounds__(32) k_boot(const __grid_constant__ GameArgs g, StateView S, u32 e, const u8* boot_pads,
                                             u32 boot_n, u32 idle_n, u8* recs, u32* fault_out) {
    extern __shared__ __align__(16) u8 smem_raw[];
    EmuShared& sh = *reinterpret_cast<EmuShared*>(smem_raw);
    u32* dtab = reinterpret_cast<u32*>(smem_raw + kDtabOff);
    u8* prg_s = smem_raw + kFramesSmem;
    const u32 lane = threadIdx.x;
    for (int i = lane; i < 256; i += 32) dtab[i] = kDecode.t[i];
    stage_prg(g.cart, prg_s, lane, 32);
    __syncwarp();
    const bool me = lane == 0;
    if (me) {
        for (int w = 0; w < kRegWords; ++w) S.regs[static_cast<u64>(w) * S.Np + e] = 0;
        for (u32 i = 0; i < kRamWords; ++i) S.ram[static_cast<u64>(i) * S.Np + e] = 0xFFFFFFFFu;
        for (u32 i = 0; i < kPrgRamWords; ++i) S.prg_ram[static_cast<u64>(i) * S.Np + e] = 0;
        for (u32 i = 0; i < kOamBytes; ++i) S.oam[static_cast<u64>(e) * kOamBytes + i] = 0;
        for (u32 i = 0; i < kNtBytes; ++i) S.nt[static_cast<u64>(e) * kNtBytes + i] = 0;
        for (u32 i = 0; i < kPalBytes; ++i) S.pal[static_cast<u64>(e) * kPalBytes + i] = 0;
        if (S.chr_ram) for (u32 i = 0; i < kChrRamBytes; ++i) S.chr_ram[static_cast<u64>(e) * kChrRamBytes + i] = 0;
        for (u32 i = 0; i < kLogBanks * kLogBankWords; ++i) S.log[static_cast<u64>(e) * kLogBanks * kLogBankWords + i] = 0;
        for (u32 i = 0; i < kNtBytes; ++i) S.snap_nt[static_cast<u64>(e) * 4 * kNtBytes + i] = 0;
        for (u32 i = 0; i < kOamBytes; ++i) S.snap_oam[static_cast<u64>(e) * 4 * kOamBytes + i] = 0;
        S.slot_bank[static_cast<u64>(e) * 4] = 0;
    }
    __syncwarp();
    Emu<BOARD> m(S, g.cart, e, lane, sh, dtab, prg_s);
    m.froze = 0;
    if (me) {
        m.stage_in();
        // paged boards keep a run-time page map (the others mirror by the header and have none); power-on registers
        // (patch:3057-3085)
        const u32 hmap = g.cart.arrangement == 1 ? kPageHorizontal : kPageVertical;
        m.ww(R_PPU2, board_paged(BOARD) ? (hmap << 24) : 0u);
        if constexpr (BOARD == kCnrom) m.cnrom_sync();
        if constexpr (BOARD == kMmc1) { m.set_mreg(0, 0x0C); m.mmc1_sync(); }
        if constexpr (BOARD == kMmc2) { m.set_mreg(6, 1); m.set_mreg(7, 1); m.mmc2_sync(); }   // both on $FE
        if constexpr (BOARD == kMmc3) {
            m.set_mreg(1, 2); m.set_mreg(2, 4); m.set_mreg(3, 5); m.set_mreg(4, 6); m.set_mreg(5, 7); m.set_mreg(7, 1);
            m.set_mreg(9, g.cart.arrangement == 1 ? 1 : 0);
            m.mmc3_sync();
        }
        m.prg_bank = 0;
        const u32 lo = m.prg_rd(0xFFFCu), hi = m.prg_rd(0xFFFDu);
        m.ww(R_PC_SP_P, (lo | (hi << 8)) | (0xFDu << 16) | (0x24u << 24));
        m.ww(R_CYC_LO, 7);
        const u64 be = 7ull + 1ull + 7ull * 428ull;   // DMC power-on: one cycle to the first bit clock, rate 0
        m.ww(R_DMC_END, static_cast<u32>(be)); m.ww(R_DMC_END + 1, 0);
        m.ww(R_DMC_EV, 0xFFFFFFFFu); m.ww(R_DMC_EV + 1, 0xFFFFFFFFu);
        m.load();
        m.fill_header(m.log_bank(0));   // both banks start from the reset state (frame_log_reset, patch:1133-1150)
        m.fill_header(m.log_bank(1));
    }
    u64 target = kVblankDot;
    u32 fault = 0;
    if (me && boot_n == 0) { m.store(); m.stage_out(); gather_record(S, e, recs, g.cart.chr == nullptr); }
    for (u32 k = 0; k < boot_n + idle_n; ++k) {
        if (me) { m.pad = k < boot_n ? boot_pads[k] : 0u; m.slot = k & 3u; }
        const u32 f = m.step_until(target, me);
        m.snapshot_frozen();
        if (me) {
            m.finish_slot();
            target += kFrameDots;
            if (f && !fault) fault = f;
            if (k + 1 >= boot_n) {
                m.store();
                m.stage_out();
                gather_record(S, e, recs + static_cast<u64>(k + 1 - boot_n) * kRecBytes, g.cart.chr == nullptr);
            }
        }
    }
    if (me) {
        m.store();
        m.stage_out();
        fault_out[0] = fault;
        fault_out[1] = static_cast<u32>(target);
        fault_out[2] = static_cast<u32>(target >> 32);
    }
}

// Canonical dump of env slot e (same bytes as the CPU oracle's oracle_dump_env).
static __global__ void k_dump(StateView S, u32 e, u32 chr_ram_cart, u8* o) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (u32 i = 0; i < kDumpBytes; ++i) o[i] = 0;
    auto R = [&](int w) { return S.regs[static_cast<u64>(w) * S.Np + e]; };
    auto p16 = [&](u32 off, u32 v) { o[off] = v & 0xFF; o[off + 1] = (v >> 8) & 0xFF; };
    auto p32 = [&](u32 off, u32 v) { for (int i = 0; i < 4; ++i) o[off + i] = (v >> (8 * i)) & 0xFF; };
    const u32 w0 = R(R_PC_SP_P), w1 = R(R_AXY_PAD);
    p16(0, w0 & 0xFFFF); o[2] = w1 & 0xFF; o[3] = (w1 >> 8) & 0xFF; o[4] = (w1 >> 16) & 0xFF; o[5] = (w0 >> 16) & 0xFF;
    o[6] = w0 >> 24; o[7] = w1 >> 24;
    p32(8, R(R_CYC_LO)); p32(12, R(R_CYC_HI));
    const u32 q0 = R(R_PPU0), q1 = R(R_PPU1), q2 = R(R_PPU2), io = R(R_IO);
    o[16] = q0 & 0xFF; o[17] = (q0 >> 8) & 0xFF; o[18] = (q0 >> 16) & 0xFF; o[19] = q0 >> 24;
    o[20] = q1 & 0xFF; o[21] = (q1 >> 8) & 0xFF; o[22] = (q1 >> 16) & 0xFF; o[23] = q1 >> 24;
    o[24] = q2 & 0xFF; o[25] = ((q2 >> 8) & 0xFF) >> 2; o[26] = io >> 24; o[27] = (q2 >> 16) & 0xFF; o[28] = q2 >> 24;
    o[29] = (io >> 16) & 0xFF; o[30] = (io >> 8) & 0xFF; o[31] = io & 0xFF;
    p32(32, R(R_FDOT)); p32(36, R(R_VT));
    p32(40, R(R_FRAME_LO)); p32(44, R(R_FRAME_HI));
    p32(48, R(R_S0)); p16(52, R(R_LOGN) & 0xFFFF);
    const u8* r8 = reinterpret_cast<const u8*>(S.ram);
    for (u32 a = 0; a < 2048; ++a) o[64 + a] = r8[((static_cast<u64>(a >> 2) * S.Np + e) << 2) | (a & 3u)];
    for (u32 a = 0; a < 2048; ++a) o[2112 + a] = S.nt[static_cast<u64>(e) * kNtBytes + a];
    for (u32 a = 0; a < 32; ++a) o[4160 + a] = S.pal[static_cast<u64>(e) * kPalBytes + a];
    for (u32 a = 0; a < 256; ++a) o[4192 + a] = S.oam[static_cast<u64>(e) * kOamBytes + a];
    for (u32 i = 0; i < 4; ++i) p32(4448 + 4 * i, R(R_MREG + i));
    for (u32 i = 0; i < 4; ++i) p32(4464 + 4 * i, R(R_PRGPG + i));
    for (u32 i = 0; i < 8; ++i) p32(4480 + 4 * i, R(R_CHRPG + i));
    p32(4512, R(R_DMC_END)); p32(4516, R(R_DMC_END + 1));
    const u32 da = R(R_DMC_A), db = R(R_DMC_B);
    p16(4520, da & 0xFFFF); o[4522] = (da >> 16) & 0xFF; o[4523] = da >> 24; o[4524] = db & 0xFF; o[4525] = (db >> 8) & 0xFF;
    p32(4528, R(R_DMC_EV)); p32(4532, R(R_DMC_EV + 1));
    const u32 shown = (q2 >> 8) & kLcBank;
    const u32* h = S.log + (static_cast<u64>(e) * kLogBanks + shown) * kLogBankWords;
    const u32 cnt = min(h[0] & ~kLogOverflow, kLogEv);
    for (u32 i = 0; i < kLogHdr + 2 * cnt; ++i) p32(4544 + 4 * i, h[i]);
    const u8* pr8 = reinterpret_cast<const u8*>(S.prg_ram);
    for (u32 a = 0; a < 8192; ++a) o[6656 + a] = pr8[((static_cast<u64>(a >> 2) * S.Np + e) << 2) | (a & 3u)];
    if (chr_ram_cart && S.chr_ram) for (u32 a = 0; a < 8192; ++a) o[14848 + a] = S.chr_ram[static_cast<u64>(e) * kChrRamBytes + a];
}

}  // namespace gr
