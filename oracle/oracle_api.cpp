// TEST INFRASTRUCTURE ONLY - liboracle_rlenv.so: the CPU oracle behind the reference environment's C-ABI
// (rl/csrc/rlenv_api.h:8-47, implemented by rl/csrc/rlenv_cpu.cpp:1-192 in the reference). Envs run under OpenMP
// `parallel for schedule(dynamic, 1)` as in rl/csrc/rlenv_cpu.cpp:35-45. Only tests/, __graft_entry__.smoke() and
// bench.py's cpu_baseline leg load this library; the product never does.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "env.hpp"
#include "../include/rlenv_api.h"   // the entry points below are compiled against the C-ABI declarations

using namespace orc;

namespace {

thread_local std::string g_error;
std::mutex g_specs_mu;
std::map<int, rw::Spec> g_specs;   // rl10 game id -> reward parameters (rl10_register_game)

// Canonical per-env machine dump shared with the product (include/rlenv_api.h, RLENV_DUMP_BYTES).
constexpr std::size_t kDumpBytes = 23040;

void put16(u8* p, u16 v) { std::memcpy(p, &v, 2); }
void put32(u8* p, u32 v) { std::memcpy(p, &v, 4); }
void put64(u8* p, u64 v) { std::memcpy(p, &v, 8); }

void dump_console(const Cart& c, const Console& m, u8* o) {
    std::memset(o, 0, kDumpBytes);
    put16(o + 0, m.pc); o[2] = m.a; o[3] = m.x; o[4] = m.y; o[5] = m.sp; o[6] = m.p; o[7] = m.pad;
    put64(o + 8, m.cycles);
    o[16] = m.ctrl; o[17] = m.mask; o[18] = m.status; o[19] = m.oam_addr; o[20] = m.nmi_pending; o[21] = m.fx;
    o[22] = m.w; o[23] = m.open_bus;
    o[24] = m.read_buffer; o[25] = static_cast<u8>(m.log_bank >> 1); o[26] = m.irq_line; o[27] = m.prg_bank; o[28] = m.mirroring;
    o[29] = m.ctl_strobe; o[30] = m.ctl_count; o[31] = m.ctl_shift;
    put32(o + 32, m.frame_dot); put16(o + 36, m.v); put16(o + 38, m.t);
    put64(o + 40, m.frame);
    put32(o + 48, m.sprite0_dot); put16(o + 52, m.log_count);
    std::memcpy(o + 64, m.ram, 2048);
    std::memcpy(o + 2112, m.nt, 2048);
    std::memcpy(o + 4160, m.pal, 32);
    std::memcpy(o + 4192, m.oam, 256);
    std::memcpy(o + 4448, m.regs, 16);
    for (int i = 0; i < 4; ++i) put32(o + 4464 + 4 * i, m.prg_page[i]);
    for (int i = 0; i < 8; ++i) put32(o + 4480 + 4 * i, m.chr_page[i]);
    put64(o + 4512, m.dmc.byte_end); put16(o + 4520, m.dmc.bytes_left); o[4522] = m.dmc.control;
    o[4523] = m.dmc.length; o[4524] = m.dmc.rate; o[4525] = m.dmc.buffer_full; put64(o + 4528, m.dmc_event);
    const u32* shown = log_bank_ptr(m, m.log_bank & 1u);
    const u32 count = (shown[0] & ~kLogOverflow) < kLogEvents ? (shown[0] & ~kLogOverflow) : kLogEvents;
    std::memcpy(o + 4544, shown, 4 * (kLogHeader + 2 * count));
    std::memcpy(o + 6656, m.prg_ram, 8192);
    if (c.chr.empty()) std::memcpy(o + 14848, m.chr_ram, 8192);
}

struct Handle {
    World w;
};

template <class F>
void each_env(World& w, F&& f) {
    const int total = w.total;
#pragma omp parallel for schedule(dynamic, 1)
    for (int k = 0; k < total; ++k) {
        std::size_t gi = 0;
        while (k >= w.games[gi].offset + w.games[gi].n) ++gi;
        f(w.games[gi], k - w.games[gi].offset);
    }
}

// Exact resume: every console (snapshot slots included) and every per-env record, then (level starts on) the
// episode start slots and each game's saved level starts, last, in the order of rl/csrc/rlenv_build.hpp:266-279,
// so a state saved without level starts is a prefix.
template <class F>
void for_each_state(World& w, F&& f) {
    for (auto& g : w.games) f(g.con.data(), g.con.size() * sizeof(Console));
    f(w.env.data(), w.env.size() * sizeof(PerEnv));
    if (!w.ep_start.empty()) {
        f(w.ep_start.data(), w.ep_start.size() * 4);
        for (auto& g : w.games) {
            f(g.lv_con.data(), g.lv_con.size() * sizeof(Console));
            f(g.lv_st.data(), g.lv_st.size() * sizeof(rw::EnvState));
            f(g.lv_target.data(), g.lv_target.size() * 8);
            f(g.lv_frame.data(), g.lv_frame.size() * 4);
            f(g.lv_deaths.data(), g.lv_deaths.size() * 4);
        }
    }
}
}  // namespace

extern "C" {

int rl10_register_game(int game_id, const double* spec, int n) {
    if (n != rw::kSpecFields || game_id < 0) { g_error = "rl10_register_game: expected 20 fields"; return 1; }
    rw::Spec s;
    std::memcpy(&s, spec, sizeof s);
    std::lock_guard<std::mutex> lock(g_specs_mu);
    g_specs[game_id] = s;
    return 0;
}

void* rlenv_create(int ngames, const int* game_ids, const std::uint8_t* const* roms, const std::size_t* rom_sizes,
                   const std::uint8_t* const* boot_pads, const std::size_t* boot_sizes, const int* n_envs,
                   std::uint64_t run_seed, int sticky, int idle_max, int dropout, int /*device*/) {
    try {
        auto h = std::make_unique<Handle>();
        World& w = h->w;
        int offset = 0;
        for (int i = 0; i < ngames; ++i) {
            Game g;
            {
                std::lock_guard<std::mutex> lock(g_specs_mu);
                auto it = g_specs.find(game_ids[i]);
                if (it == g_specs.end() || it->second.reader != 1.0)
                    throw std::runtime_error("game id " + std::to_string(game_ids[i]) +
                                             ": the oracle runs registered synthetic games only");
                g.spec = it->second;
            }
            g.cart = parse_ines(roms[i], rom_sizes[i]);
            g.game_id = game_ids[i];
            g.n = n_envs[i];
            g.offset = offset;
            offset += g.n;
            g.start_ok = g.spec.start_ok != 0.0;
            g.select_ok = g.spec.select_ok != 0.0;
            Console boot;
            cold_reset(g.cart, boot);
            u64 target = kVblankDot;
            for (std::size_t k = 0; k < boot_sizes[i]; ++k) {
                boot.pad = boot_pads[i][k];
                if (step_until(g.cart, boot, target) != 0)
                    throw std::runtime_error("emulator fault during boot of game " + std::to_string(game_ids[i]));
                target += kFrameDots;
            }
            g.con.assign(static_cast<std::size_t>(g.n) + 1, boot);
            g.tmpl_target = target;
            g.idle_tmpl = idle_max > 0 ? idle_max : 0;
            for (int k = 1; k <= g.idle_tmpl; ++k) {
                boot.pad = 0;
                if (step_until(g.cart, boot, target) != 0)
                    throw std::runtime_error("emulator fault in idle frames of game " + std::to_string(game_ids[i]));
                target += kFrameDots;
                g.idle_snap.push_back(boot);
            }
            w.games.push_back(std::move(g));
        }
        w.total = offset;
        w.env.assign(static_cast<std::size_t>(offset), PerEnv{});
        for (auto& pe : w.env) pe.episode = 0xFFFFFFFFu;
        w.run_seed = run_seed;
        w.sticky = sticky;
        w.idle_max = idle_max;
        w.dropout = dropout;
        return h.release();
    } catch (const std::exception& ex) {
        g_error = ex.what();
        return nullptr;
    }
}

int rlenv_num_envs(void* h) { return static_cast<Handle*>(h)->w.total; }
void rlenv_set_episode_level_end(void* h, int level) { static_cast<Handle*>(h)->w.episode_level_end = level; }
void rlenv_set_no_render(void* h, int v) { static_cast<Handle*>(h)->w.no_render = v; }

void rlenv_bind(void* h, const std::int16_t* actions, std::uint8_t* obs, std::uint8_t* emph, float* reward,
                std::uint8_t* done, std::uint8_t* masks, std::uint8_t* timeline, std::uint8_t* pads,
                std::uint32_t* events, float* info) {
    Outputs& o = static_cast<Handle*>(h)->w.out;
    o.actions = actions; o.obs = obs; o.emph = emph; o.reward = reward; o.done = done; o.masks = masks;
    o.timeline = timeline; o.pads = pads; o.events = events; o.info = info;
}
void rlenv_bind_parts(void* h, float* parts) { static_cast<Handle*>(h)->w.out.parts = parts; }
void rlenv_bind_obs(void* h, std::uint8_t* obs, std::uint8_t* emph) {
    Outputs& o = static_cast<Handle*>(h)->w.out;
    o.obs = obs;
    o.emph = emph;
}

int rlenv_start(void* h, void*) {
    World& w = static_cast<Handle*>(h)->w;
    each_env(w, [&](Game& g, int e) { env_start(g, w, e); });
    return 0;
}

int rlenv_step(void* h, void*) {
    World& w = static_cast<Handle*>(h)->w;
    each_env(w, [&](Game& g, int e) { env_step(g, w, e); });
    for (auto& g : w.games) archive(g, w);   // after every env's decision, as rl/csrc/rlenv_cpu.cpp:100-116
    return 0;
}

// ---- level starts and places (rl/csrc/rlenv_cpu.cpp:119-170, rl/csrc/rlenv_build.hpp:212-252)

int rlenv_enable_places(void* h, int cap, int levels) {
    World& w = static_cast<Handle*>(h)->w;
    if (!w.ep_start.empty() || cap <= 0 || levels <= 0 || levels > cap) {
        g_error = "level starts: enable once, 0 < levels <= cap";
        return 1;
    }
    for (auto& g : w.games) {
        g.lv_cap = cap;
        g.lv_levels = levels;
        g.lv_con.assign(static_cast<std::size_t>(cap), Console{});
        g.lv_st.assign(static_cast<std::size_t>(cap), rw::EnvState{});
        g.lv_target.assign(static_cast<std::size_t>(cap), 0);
        g.lv_frame.assign(static_cast<std::size_t>(cap), 0);
        g.lv_deaths.assign(static_cast<std::size_t>(cap), -1);
        g.lv_claim.assign(static_cast<std::size_t>(cap), ~0ull);
        g.lv_cdf.assign(static_cast<std::size_t>(cap), 0);
    }
    w.ep_start.assign(static_cast<std::size_t>(w.total), -1);
    return 0;
}
int rlenv_enable_level_starts(void* h, int cap) { return rlenv_enable_places(h, cap, cap); }
void rlenv_set_level_plan(void* h, int gi, double p, const std::uint32_t* cdf) {
    Game& g = static_cast<Handle*>(h)->w.games[static_cast<std::size_t>(gi)];
    if (g.lv_cap == 0) return;
    g.lv_thresh = static_cast<u32>(p <= 0.0 ? 0.0 : p >= 1.0 ? 4294967295.0 : p * 4294967296.0);
    g.lv_weighted = cdf != nullptr;
    if (cdf) std::memcpy(g.lv_cdf.data(), cdf, static_cast<std::size_t>(g.lv_cap) * 4);
}
void rlenv_bind_start(void* h, std::int32_t* p) { static_cast<Handle*>(h)->w.out.start_out = p; }
void rlenv_bind_level(void* h, std::int32_t* p) { static_cast<Handle*>(h)->w.out.level_out = p; }
void rlenv_bind_progress(void* h, float* p) { static_cast<Handle*>(h)->w.out.progress_out = p; }
int rlenv_level_deaths(void* h, int gi, std::int32_t* out, void*) {
    const Game& g = static_cast<Handle*>(h)->w.games[static_cast<std::size_t>(gi)];
    if (g.lv_cap) std::memcpy(out, g.lv_deaths.data(), static_cast<std::size_t>(g.lv_cap) * 4);
    return 0;
}
int rlenv_place_save(void* h, int gi, const std::int32_t* env_idx, const std::int32_t* slot_idx, int count, void*) {
    World& w = static_cast<Handle*>(h)->w;
    Game& g = w.games[static_cast<std::size_t>(gi)];
    if (g.lv_cap == 0) return 0;
    for (int i = 0; i < count; ++i) place_save(g, w, env_idx[i], slot_idx[i]);
    return 0;
}
int rlenv_place_copy(void* h, int gi, const std::int32_t* src, const std::int32_t* dst, int count, void*) {
    Game& g = static_cast<Handle*>(h)->w.games[static_cast<std::size_t>(gi)];
    for (int i = 0; i < count; ++i)
        if (src[i] < 0 || dst[i] < 0 || src[i] >= g.lv_cap || dst[i] >= g.lv_cap) { g_error = "place_copy: bad slot"; return 1; }
    for (int i = 0; i < count; ++i) {
        const std::size_t a = static_cast<std::size_t>(src[i]), b = static_cast<std::size_t>(dst[i]);
        g.lv_con[b] = g.lv_con[a]; g.lv_st[b] = g.lv_st[a]; g.lv_target[b] = g.lv_target[a];
        g.lv_frame[b] = g.lv_frame[a]; g.lv_deaths[b] = g.lv_deaths[a];
    }
    return 0;
}
void rlenv_level_layout(void* h, int gi, std::uint32_t* out) {
    const Game& g = static_cast<Handle*>(h)->w.games[static_cast<std::size_t>(gi)];
    out[0] = static_cast<u32>(sizeof(Console)); out[1] = 0; out[2] = static_cast<u32>(sizeof(rw::EnvState));
    out[3] = static_cast<u32>(g.lv_cap); out[4] = static_cast<u32>(g.lv_levels);
}

std::size_t rlenv_state_bytes(void* h) {
    std::size_t n = 0;
    for_each_state(static_cast<Handle*>(h)->w, [&](void*, std::size_t b) { n += b; });
    return n;
}
int rlenv_save(void* h, std::uint8_t* out, void*) {
    for_each_state(static_cast<Handle*>(h)->w, [&](void* p, std::size_t b) { std::memcpy(out, p, b); out += b; });
    return 0;
}
int rlenv_load(void* h, const std::uint8_t* in, void*) {
    for_each_state(static_cast<Handle*>(h)->w, [&](void* p, std::size_t b) { std::memcpy(p, in, b); in += b; });
    return 0;
}

const char* rlenv_error() { return g_error.c_str(); }
void rlenv_destroy(void* h) { delete static_cast<Handle*>(h); }

// ---------------------------------------------------------------- oracle-only test exports

std::size_t oracle_dump_bytes() { return kDumpBytes; }

// Canonical machine state of global env `ge` (see include/rlenv_api.h for the layout).
int oracle_dump_env(void* h, int ge, std::uint8_t* out) {
    World& w = static_cast<Handle*>(h)->w;
    if (ge < 0 || ge >= w.total) { g_error = "dump: bad env"; return 1; }
    std::size_t gi = 0;
    while (ge >= w.games[gi].offset + w.games[gi].n) ++gi;
    const Game& g = w.games[gi];
    dump_console(g.cart, g.con[ge - g.offset], out);
    return 0;
}

// Per-env RL scalars: target, ep_frame, episode, fault, sticky_ctr.
// Both frame-log banks of global env ge (2 x 528 words: the shown one first, then the other, which after a decision
// still holds the frame before the shown one; nothing runs between a frame's vblank stop and the next decision).
int oracle_log_banks(void* h, int ge, std::uint32_t* out) {
    World& w = static_cast<Handle*>(h)->w;
    if (ge < 0 || ge >= w.total) { g_error = "log banks: bad env"; return 1; }
    std::size_t gi = 0;
    while (ge >= w.games[gi].offset + w.games[gi].n) ++gi;
    const Console& m = w.games[gi].con[ge - w.games[gi].offset];
    std::memcpy(out, log_bank_ptr(m, m.log_bank & 1u), 4 * kLogBank);
    std::memcpy(out + kLogBank, log_bank_ptr(m, (m.log_bank & 1u) ^ 1u), 4 * kLogBank);
    return 0;
}

int oracle_env_scalars(void* h, int ge, std::uint64_t* out) {
    World& w = static_cast<Handle*>(h)->w;
    const PerEnv& pe = w.env[ge];
    out[0] = pe.target; out[1] = pe.ep_frame; out[2] = pe.episode; out[3] = pe.fault; out[4] = pe.sticky_ctr;
    return 0;
}

// A standalone console for emulator-level tests: power-on, then `frames` frames with the given pads; dumps after.
int oracle_run_frames(const std::uint8_t* rom, std::size_t rom_size, const std::uint8_t* pads, int frames,
                      std::uint8_t* dump_out, std::uint8_t* obs_out, std::uint8_t* emph_out, std::uint32_t* faults) {
    try {
        const Cart c = parse_ines(rom, rom_size);
        Console m;
        cold_reset(c, m);
        u64 target = kVblankDot;
        for (int f = 0; f < frames; ++f) {
            m.pad = pads[f];
            faults[f] = step_until(c, m, target);
            target += kFrameDots;
            if (obs_out) render_obs(c, m, obs_out + static_cast<std::size_t>(f) * kObsPixels,
                                    emph_out + static_cast<std::size_t>(f) * kObsH);
            if (dump_out) dump_console(c, m, dump_out + static_cast<std::size_t>(f) * kDumpBytes);
        }
        return 0;
    } catch (const std::exception& ex) {
        g_error = ex.what();
        return 1;
    }
}

// Per-frame cost split on one thread, the reference's method (rl/bench/split_cpu.cpp:1-30): the boot frames, then
// `frames` frames with LCG pads (x = x * 1103515245 + 12345, pad = (x >> 16) & 0xF3), each timed as emulating the
// frame (step_until) and drawing it (render_obs). out[0] = emulate us / frame, out[1] = draw us / frame.
int oracle_split_frames(const std::uint8_t* rom, std::size_t rom_size, const std::uint8_t* boot, int boot_n, int frames,
                        double* out) {
    try {
        const Cart c = parse_ines(rom, rom_size);
        Console m;
        cold_reset(c, m);
        u64 target = kVblankDot;
        for (int f = 0; f < boot_n; ++f) {
            m.pad = boot[f];
            step_until(c, m, target);
            target += kFrameDots;
        }
        std::vector<std::uint8_t> pix(kObsPixels), em(kObsH);
        double te = 0, tr = 0;
        unsigned x = 1;
        for (int i = 0; i < frames; ++i) {
            x = x * 1103515245u + 12345u;
            m.pad = static_cast<u8>((x >> 16) & 0xF3);
            const auto t0 = std::chrono::steady_clock::now();
            step_until(c, m, target);
            target += kFrameDots;
            const auto t1 = std::chrono::steady_clock::now();
            render_obs(c, m, pix.data(), em.data());
            const auto t2 = std::chrono::steady_clock::now();
            te += std::chrono::duration<double>(t1 - t0).count();
            tr += std::chrono::duration<double>(t2 - t1).count();
        }
        out[0] = 1e6 * te / frames;
        out[1] = 1e6 * tr / frames;
        return 0;
    } catch (const std::exception& ex) {
        g_error = ex.what();
        return 1;
    }
}

// reward10 on a RAM trace with a registered spec (the shape of the reference's rl10_replay, host_api.cpp:13-30).
int oracle_reward_replay(int game_id, const std::uint8_t* ram, int n, const int* frames, double* reward,
                         std::uint8_t* done, std::uint32_t* events, int* event_level, int* deaths,
                         std::uint8_t* end_reason, double* parts) {
    rw::Spec spec;
    {
        std::lock_guard<std::mutex> lock(g_specs_mu);
        auto it = g_specs.find(game_id);
        if (it == g_specs.end()) { g_error = "unregistered game"; return 1; }
        spec = it->second;
    }
    rw::EnvState e{};
    for (int i = 0; i < n; ++i) {
        const rw::Update u = rw::update(spec, ram + static_cast<std::size_t>(i) * 2048, frames[i], e);
        reward[i] = u.reward;
        done[i] = u.done ? 1 : 0;
        events[i] = u.events;
        event_level[i] = u.event_level;
        deaths[i] = e.deaths;
        end_reason[i] = e.end_reason;
        if (parts) for (int k = 0; k < rw::kParts; ++k) parts[i * rw::kParts + k] = u.part[k];
    }
    return 0;
}

// Controller tables in the layout of the reference's host_api.cpp:35-67 (checked against it).
void oracle_pad_table(std::uint8_t* out) {
    for (int id = 0; id < ctl::kMoves; ++id)
        for (int f = 0; f < 2; ++f) out[2 * id + f] = ctl::pad_byte(ctl::unpack(id), static_cast<u64>(f));
}
void oracle_legal_table(int start_ok, int select_ok, std::uint8_t* out, std::int32_t* rest) {
    for (int d = -1; d < ctl::kDropInputs; ++d) {
        const auto k = ctl::legal(d, start_ok != 0, select_ok != 0);
        for (int id = 0; id < ctl::kMoves; ++id) {
            const auto m = ctl::unpack(id);
            const bool ok = ((k.dpad >> m.dpad) & 1) && ((k.a >> m.a) & 1) && ((k.b >> m.b) & 1) &&
                            ((k.start >> m.start) & 1) && ((k.select >> m.select) & 1);
            out[(d + 1) * ctl::kMoves + id] = ok ? 1 : 0;
            rest[(d + 1) * ctl::kMoves + id] = ctl::pack(ctl::restrict_move(m, d, start_ok != 0, select_ok != 0));
        }
    }
}
void oracle_schedule(std::uint64_t seed, int enabled, int n, std::int8_t* dropped, std::uint8_t* timelines) {
    ctl::Dropout s;
    ctl::dropout_reset(s, seed, enabled != 0);
    for (int t = 0; t < n; ++t) {
        dropped[t] = static_cast<std::int8_t>(ctl::dropped_now(s));
        if (timelines) ctl::timeline(s, timelines + static_cast<std::size_t>(t) * ctl::kDropInputs * ctl::kTimeline);
        ctl::dropout_advance(s, enabled != 0);
    }
}
std::uint64_t oracle_episode_seed(std::uint64_t run_seed, std::uint32_t env, std::uint64_t episode) {
    return ctl::episode_seed(run_seed, env, episode);
}

}  // extern "C"
