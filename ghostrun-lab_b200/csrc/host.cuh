// Host-side runtime shared by the library's translation units: device memory, cartridge parsing, the per-game
// launch sequence and the boot run. The board-specialised templates (launch_game / boot_game) are instantiated
// once per board in board_*.cu, so the four emulator specialisations compile in parallel.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "envcore.cuh"

namespace gr {

inline void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct DevMem {
    std::vector<void*> blocks;
    std::vector<std::pair<void*, std::size_t>> state;   // (ptr, bytes) saved by rlenv_save, in order
    void* alloc(std::size_t n, bool saved = false) {
        void* p = nullptr;
        ck(cudaMalloc(&p, n ? n : 16), "cudaMalloc");
        ck(cudaMemset(p, 0, n ? n : 16), "cudaMemset");
        blocks.push_back(p);
        if (saved) state.emplace_back(p, n);
        return p;
    }
    template <class T> T* allocn(std::size_t count, bool saved = false) { return static_cast<T*>(alloc(sizeof(T) * count, saved)); }
    ~DevMem() { for (void* p : blocks) cudaFree(p); }
};

// Device arrays of a StateView for Np env slots (env-minor words, env-major bytes, 4 presentation slots each).
inline StateView alloc_state_view(DevMem& M, u32 Np, bool chr_ram, bool saved) {
    StateView S{};
    S.Np = Np;
    S.regs = M.allocn<u32>(static_cast<std::size_t>(kRegWords) * Np, saved);
    S.ram = M.allocn<u32>(static_cast<std::size_t>(kRamWords) * Np, saved);
    S.prg_ram = M.allocn<u32>(static_cast<std::size_t>(kPrgRamWords) * Np, saved);
    S.oam = M.allocn<u8>(static_cast<std::size_t>(kOamBytes) * Np, saved);
    S.nt = M.allocn<u8>(static_cast<std::size_t>(kNtBytes) * Np, saved);
    S.pal = M.allocn<u8>(static_cast<std::size_t>(kPalBytes) * Np, saved);
    S.chr_ram = chr_ram ? M.allocn<u8>(static_cast<std::size_t>(kChrRamBytes) * Np, saved) : nullptr;
    S.log = M.allocn<u32>(static_cast<std::size_t>(kLogBanks) * kLogBankWords * Np, saved);
    S.snap_nt = M.allocn<u8>(static_cast<std::size_t>(4) * kNtBytes * Np, saved);
    S.snap_oam = M.allocn<u8>(static_cast<std::size_t>(4) * kOamBytes * Np, saved);
    S.snap_chr = chr_ram ? M.allocn<u8>(static_cast<std::size_t>(4) * kChrRamBytes * Np, saved) : nullptr;
    S.slot_bank = M.allocn<u8>(static_cast<std::size_t>(4) * Np, saved);
    if (chr_ram && saved) {   // the main state only (scratch views copy every frame)
        S.chr_shared = M.allocn<u8>(static_cast<std::size_t>(kChrRamBytes) * Np, saved);
        S.chr_ref = M.allocn<u8>(static_cast<std::size_t>(4) * Np, saved);
    }
    return S;
}

// iNES 1.0 header -> board description (the product's own parser; rl/csrc/rlenv_build.hpp:36-84 uses NeSLE's).
struct HostCart {
    std::vector<u8> prg, chr;
    u32 board = kNrom, arrangement = 0, bank_mask = 0, fixed_base = 0, prg_page_mask = 0, chr_page_mask = 0;
};

inline HostCart parse_rom(const u8* rom, std::size_t n) {
    if (n < 16 || std::memcmp(rom, "NES\x1a", 4) != 0) throw std::runtime_error("not an iNES image");
    const std::size_t prg_bytes = static_cast<std::size_t>(rom[4]) * 16384, chr_bytes = static_cast<std::size_t>(rom[5]) * 8192;
    const u32 mapper = (rom[6] >> 4) | (rom[7] & 0xF0u);
    const std::size_t base = 16 + ((rom[6] & 4) ? 512 : 0);
    if (prg_bytes == 0 || base + prg_bytes + chr_bytes > n) throw std::runtime_error("truncated iNES image");
    HostCart c;
    std::size_t padded = 1;
    while (padded < prg_bytes) padded <<= 1;
    c.prg.assign(padded, 0);
    std::memcpy(c.prg.data(), rom + base, prg_bytes);
    c.chr.assign(rom + base + prg_bytes, rom + base + prg_bytes + chr_bytes);
    c.arrangement = (rom[6] & 8) ? 2u : (rom[6] & 1) ? 0u : 1u;
    const bool pow2 = (prg_bytes & (prg_bytes - 1)) == 0;
    if (mapper == 0) {
        if ((prg_bytes != 16384 && prg_bytes != 32768) || chr_bytes == 0) throw std::runtime_error("NROM needs 16/32 KB PRG and CHR ROM");
        c.board = kNrom;
    } else if (mapper == 2) {
        if (prg_bytes < 32768 || !pow2) throw std::runtime_error("UxROM PRG must be a power of two >= 32 KB");
        c.board = kUxrom;
        c.bank_mask = static_cast<u32>(prg_bytes / 16384 - 1);
        c.fixed_base = static_cast<u32>(prg_bytes - 16384);
    } else if (mapper == 3) {   // CNROM (patch:4007-4030): PRG pages 0-3 mapped, CHR ROM in 8 KB banks
        if (prg_bytes < 16384 || prg_bytes > 512 * 1024 || !pow2 || chr_bytes == 0 || (chr_bytes & (chr_bytes - 1)) ||
            chr_bytes > 256 * 1024)
            throw std::runtime_error("unsupported CNROM image size (PRG 16-512 KB, a power-of-two CHR ROM up to 256 KB)");
        c.board = kCnrom;
        c.prg_page_mask = static_cast<u32>(prg_bytes / 8192 - 1);
        c.chr_page_mask = static_cast<u32>(chr_bytes / 1024 - 1);
    } else if (mapper == 9) {   // MMC2 (patch:4007-4030): 8 KB PRG pages, CHR ROM only, at most 256 KB
        if (prg_bytes < 32768 || prg_bytes > 512 * 1024 || !pow2 || chr_bytes == 0 || (chr_bytes & (chr_bytes - 1)) ||
            chr_bytes > 256 * 1024)
            throw std::runtime_error("unsupported MMC2 image size");
        c.board = kMmc2;
        c.prg_page_mask = static_cast<u32>(prg_bytes / 8192 - 1);
        c.chr_page_mask = static_cast<u32>(chr_bytes / 1024 - 1);
    } else if (mapper == 1 || mapper == 4) {
        const std::size_t cb = chr_bytes ? chr_bytes : 8192;
        if (prg_bytes < 32768 || prg_bytes > 512 * 1024 || !pow2 || (cb & (cb - 1)) || cb > 256 * 1024)
            throw std::runtime_error("unsupported MMC1/MMC3 image size");
        c.board = mapper == 1 ? kMmc1 : kMmc3;
        c.prg_page_mask = static_cast<u32>(prg_bytes / 8192 - 1);
        c.chr_page_mask = static_cast<u32>(cb / 1024 - 1);
    } else {
        throw std::runtime_error("unsupported mapper " + std::to_string(mapper) + " (supported: 0 NROM, 1 MMC1, 2 UxROM, 3 CNROM, 4 MMC3, 9 MMC2)");
    }
    return c;
}

// CHR ROM as 4-bit-per-pixel rows (render.cuh): chrx[row * 512 + tile], first 8 KB.
inline std::vector<u32> expand_chr(const std::vector<u8>& chr) {
    std::vector<u32> out(4096, 0);
    auto spread = [](u32 b) { u32 r = 0; for (int k = 0; k < 8; ++k) r |= ((b >> (7 - k)) & 1u) << (4 * k); return r; };
    for (u32 tile = 0; tile < 512; ++tile)
        for (u32 row = 0; row < 8; ++row) {
            const u32 lo = chr[(tile * 16 + row) % chr.size()], hi = chr[(tile * 16 + row + 8) % chr.size()];
            out[row * 512 + tile] = spread(lo) | (spread(hi) << 1);
        }
    return out;
}

// Per-kernel device time on the launching stream (CUDA events around each launch), for the benchmark's roofline
// and launch count. Off by default: no events are recorded.
enum KernelKind : int { kKFrames = 0, kKRender, kKFinish, kKRestart, kKRestartRender, kKPack6, kKinds };

struct KTimer {
    bool on = false;
    unsigned mask = ~0u;   // kinds timed while on (bit k = kind k)
    double ms[kKinds] = {};
    unsigned long long launches[kKinds] = {};
    unsigned long long total_launches = 0;
    std::vector<cudaEvent_t> pool;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> pending;
    cudaEvent_t cur_a = nullptr;
    cudaEvent_t take() {
        if (pool.empty()) { cudaEvent_t e; ck(cudaEventCreate(&e), "event"); return e; }
        cudaEvent_t e = pool.back(); pool.pop_back(); return e;
    }
    void begin(int kind, cudaStream_t s) {
        ++total_launches;
        ++launches[kind];
        if (!on || !((mask >> kind) & 1u)) { cur_a = nullptr; return; }
        cur_a = take();
        ck(cudaEventRecord(cur_a, s), "event");
    }
    void end(int kind, cudaStream_t s) {
        if (!on || !cur_a) return;
        cudaEvent_t b = take();
        ck(cudaEventRecord(b, s), "event");
        pending.push_back({kind, {cur_a, b}});
    }
    void collect() {
        for (auto& p : pending) {
            float t = 0;
            ck(cudaEventSynchronize(p.second.second), "event sync");
            ck(cudaEventElapsedTime(&t, p.second.first, p.second.second), "elapsed");
            ms[p.first] += t;
            pool.push_back(p.second.first);
            pool.push_back(p.second.second);
        }
        pending.clear();
    }
    void reset() { collect(); for (int k = 0; k < kKinds; ++k) { ms[k] = 0; launches[k] = 0; } total_launches = 0; }
    ~KTimer() { for (auto e : pool) cudaEventDestroy(e); for (auto& p : pending) { cudaEventDestroy(p.second.first); cudaEventDestroy(p.second.second); } }
};

// A sub-range of one game's envs and / or other picture outputs (rlenv_step_game / rlenv_step_range).
struct Range {
    int start = 0, count = -1;
    u8* obs = nullptr;
    u8* emph = nullptr;
};

// Where a launch forks its restart work: a side stream, the event it waits for on the caller's stream, and the event
// the caller's stream waits for at the join.
struct Side {
    cudaStream_t stream;
    cudaEvent_t fork, done;
};


struct Game {
    int game_id = 0;
    int index = 0;        // position in Env::games (its restart counter)
    GameArgs g{};
    bool chrx_smem = false;
};

struct Env {
    DevMem mem;
    int device = 0;
    int total = 0;
    int lv_cap = 0, lv_levels = 0;   // level starts (rlenv_enable_places); 0 = off
    u32 Np = 0;
    std::vector<Game> games;
    EnvArgs A{};
    KTimer* timer = nullptr;
    bool chr_ram_any = false;
    cudaEvent_t ev = nullptr;
    // Per game: a main stream (games run concurrently, as the reference's one stream per game, rl/csrc/rlenv.cu:
    // 173-182) and a highest-priority side stream for its restart work; events to fork from the caller's stream and
    // join back. A one-game env runs its main work on the caller's stream itself.
    std::vector<cudaStream_t> gmain, gside;
    std::vector<cudaEvent_t> gfork, gmain_done, gside_done;
    cudaEvent_t ev_begin = nullptr;
    // Ranges (rlenv_step_range) fork their restart work onto a side stream of the CALLER's stream, created on first
    // use, so that parts of one game stepped on different caller streams overlap instead of meeting on the game's
    // side stream. Each range lists its restarting envs in its own slice of the list, with its own counter.
    struct CallerSide { cudaStream_t caller, side; cudaEvent_t fork, done; };
    std::vector<CallerSide> range_sides;
    int side_priority = 0;
    ~Env() {
        for (auto& c : range_sides) { cudaEventDestroy(c.fork); cudaEventDestroy(c.done); cudaStreamDestroy(c.side); }
        if (ev) cudaEventDestroy(ev);
        if (ev_begin) cudaEventDestroy(ev_begin);
        for (auto e : gfork) cudaEventDestroy(e);
        for (auto e : gmain_done) cudaEventDestroy(e);
        for (auto e : gside_done) cudaEventDestroy(e);
        for (auto q : gmain) cudaStreamDestroy(q);
        for (auto q : gside) cudaStreamDestroy(q);
        delete timer;
    }
};

inline void check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// One game slice's decision (or start) on the caller's stream `s`, with the restart work forked onto the env's
// high-priority side stream so it overlaps the main render:
//   s:    [list reset] k_frames -> k_finish --fork--> k_render, k_render_seq (envs not restarting) .. join (join_side)
//   side:                          k_restore -> [k_archive] -> k_frames(restart) -> k_render, k_render_seq (restart)
// (k_restore copies a boot restart's whole outcome from its restart template when there is one; the restart frames
// and drawing then leave that env out)
// Games run on their own stream pairs, concurrently (launch_all).
// k_finish decides the episode ends and lists the restarting envs; the main render leaves them out (their outputs
// are the new episode's first frames, drawn by the restart pass), so the two branches touch disjoint envs. The level
// archive reads the slots only in k_finish (the pick) and k_restore (the copy), so it saves after both, as the
// reference's k_archive after k_finish (rl/csrc/rlenv.cu:165-166).
// Launch phases (launch_all issues each phase for every game before the next, so kernels of different games that
// share a hardware work queue queue up behind work they would wait for anyway).
enum : u32 { kPhFrames = 1, kPhFinish = 2, kPhRender = 4, kPhRestart = 8, kPhAll = 15 };

template <u32 B>
void launch_game(const Env& env, const Game& gm, bool start, cudaStream_t s, const Side& sd, const Range& rg,
                 u32 phases) {
    cudaStream_t side = sd.stream;
    GameArgs g = gm.g;
    const EnvArgs& A0 = env.A;
    EnvArgs A = A0;
    if (rg.obs) { A.obs = rg.obs; A.emph = rg.emph; }
    if (rg.count >= 0) { g.e0 = gm.g.e0 + static_cast<u32>(rg.start); g.n = static_cast<u32>(rg.count); }
    // this game's (or this range's) restart list and count: a range lists into its own slice, counter after the games'
    const bool ranged = rg.count >= 0;
    A.list = A0.list + gm.g.game_e0 + (ranged ? static_cast<u32>(rg.start) : 0u);
    A.list_count = A0.list_count + (ranged ? env.games.size() + 1 + gm.g.game_e0 + static_cast<u32>(rg.start)
                                           : static_cast<std::size_t>(gm.index));
    const u32 n = g.n;
    if (n == 0) return;
    const u32 tb = 128;
    RenderArgs R{};
    R.cart = g.cart;
    R.st = A.st;
    R.obs = A.obs;
    R.emph = A.emph;
    R.packed = A.packed;
    R.seqf = A.render_seq;
    R.stats = A.render_stats;
    R.e0 = g.e0;
    R.count = n;
    R.frames = kFramesPerDecision;
    R.chrx_smem = gm.chrx_smem ? 1u : 0u;
    R.one = 1u;
    const std::size_t smem = render_smem(gm.chrx_smem), seq_smem = render_seq_smem(gm.chrx_smem);
    KTimer& T = *env.timer;
    if (phases & kPhFrames) {
        ck(cudaMemsetAsync(A.list_count, 0, 4, s), "list reset");
        if (!start) {
            T.begin(kKFrames, s);
            k_frames<B><<<frames_blocks(n), 32 * kFramesWarps, frames_smem(g.cart), s>>>(g, A, 0);
            T.end(kKFrames, s);
            check_launch("k_frames");
        }
    }
    if (phases & kPhFinish) {
        T.begin(kKFinish, s);
        k_finish<<<(n + tb - 1) / tb, tb, 0, s>>>(g, A, start ? 1 : 0);
        T.end(kKFinish, s);
        check_launch("k_finish");
        ck(cudaEventRecord(sd.fork, s), "fork");
    }
    if ((phases & kPhRender) && !start && !A.no_render) {
        R.list = nullptr;
        R.skip = A.done;
        const u32 items = n * R.frames;
        // a block per kRenderWarps frames, no cap: the last wave's tail is one frame, not one block of several
        // (measured: 1.80 -> 1.75 ms per decision against 4 waves of 296 blocks; 2 waves were slower)
        const u32 blocks = (items + kRenderWarps - 1) / kRenderWarps;
        T.begin(kKRender, s);
        k_render<B><<<blocks, 32 * kRenderWarps, smem, s>>>(R);
        T.end(kKRender, s);
        check_launch("k_render");
        T.begin(kKRender, s);
        k_render_seq<B><<<std::min<u32>(blocks, 148u * 2u), 32 * kRenderWarps, seq_smem, s>>>(R);
        T.end(kKRender, s);
        check_launch("k_render_seq");
    }
    if (!(phases & kPhRestart)) return;
    ck(cudaStreamWaitEvent(side, sd.fork, 0), "fork");
    const u32 wb = frames_blocks(n);
    if (g.lv_cap > 0 && g.lv_idle_n > 0) {   // idle chains of the slots that changed, before the restores use them
        T.begin(kKFinish, side);
        k_chain<B><<<g.lv_cap, 32, frames_smem(g.cart), side>>>(g);
        T.end(kKFinish, side);
        check_launch("k_chain");
    }
    T.begin(kKFinish, side);
    k_restore<<<start ? std::min<u32>(n, 148u * 8u) : 148u, 128, 0, side>>>(g, A);
    T.end(kKFinish, side);
    check_launch("k_restore");
    if (!start && g.lv_cap > 0) {   // level-start saves: after the pick and copy of every restarting env
        T.begin(kKFinish, side);
        k_archive<<<g.lv_levels, 128, 0, side>>>(g, A);
        T.end(kKFinish, side);
        check_launch("k_archive");
    }
    const u32 rb = start ? wb : std::min<u32>(wb, std::max<u32>(148u, 148u * (32u / kEnvsPerWarp) / kFramesWarps));
    T.begin(kKRestart, side);
    k_frames<B><<<rb, 32 * kFramesWarps, frames_smem(g.cart), side>>>(g, A, 1);
    T.end(kKRestart, side);
    check_launch("k_frames restart");
    if (!A.no_render) {
        R.list = A.list;
        R.list_count = A.list_count;
        R.skip = A.tm_used;   // restarts copied from a template have their first observation already
        const u32 blocks = start ? std::min<u32>((n * R.frames + kRenderWarps - 1) / kRenderWarps, 148u * 2u * 4u) : 148u;
        T.begin(kKRestartRender, side);
        k_render<B><<<blocks, 32 * kRenderWarps, smem, side>>>(R);
        T.end(kKRestartRender, side);
        check_launch("k_render restart");
        T.begin(kKRestartRender, side);
        k_render_seq<B><<<std::min<u32>(blocks, 148u * 2u), 32 * kRenderWarps, seq_smem, side>>>(R);
        T.end(kKRestartRender, side);
        check_launch("k_render_seq restart");
    }
}

// Game gi's own side stream (whole-game launches).
inline Side game_side(const Env& env, int gi) { return Side{env.gside[gi], env.gfork[gi], env.gside_done[gi]}; }

// The caller's stream waits for the side stream's restart work.
inline void join_side(const Side& sd, cudaStream_t s) {
    ck(cudaEventRecord(sd.done, sd.stream), "join");
    ck(cudaStreamWaitEvent(s, sd.done, 0), "join");
}

template <u32 B>
void boot_game(Env& env, Game& gm, const u8* pads, std::size_t npads, int idle_max, u32 slot) {
    u8* dpads = env.mem.allocn<u8>(npads + 1);
    if (npads) ck(cudaMemcpy(dpads, pads, npads, cudaMemcpyHostToDevice), "boot pads");
    u32* fault = env.mem.allocn<u32>(4);
    const u32 idle = idle_max > 0 ? static_cast<u32>(idle_max) : 0u;
    u8* recs = env.mem.allocn<u8>(static_cast<std::size_t>(idle + 1) * kRecBytes);
    ck(cudaFuncSetAttribute(k_frames<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFramesSmem + kPrgStageMax)),
       "smem attr");
    ck(cudaFuncSetAttribute(k_boot<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFramesSmem + kPrgStageMax)),
       "smem attr");
    ck(cudaFuncSetAttribute(k_chain<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kFramesSmem + kPrgStageMax)),
       "smem attr");
    ck(cudaFuncSetAttribute(k_render_seq<B>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(render_seq_smem(gm.chrx_smem))), "smem attr");
    ck(cudaFuncSetAttribute(k_render<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(render_smem(gm.chrx_smem))),
       "smem attr");
    k_boot<B><<<1, 32, frames_smem(gm.g.cart)>>>(gm.g, env.A.st, slot, dpads, static_cast<u32>(npads), idle, recs, fault);
    check_launch("k_boot");
    u32 hf[4] = {0, 0, 0, 0};
    ck(cudaMemcpy(hf, fault, 16, cudaMemcpyDeviceToHost), "boot");
    if (hf[0]) {
        char buf[96];
        std::snprintf(buf, sizeof buf, "emulator fault during boot of game %d (pc<<8|op = 0x%06x)", gm.game_id, hf[0]);
        throw std::runtime_error(buf);
    }
    gm.g.recs = recs;
    gm.g.idle_tmpl = idle;
    {   // restart templates, taken after rlenv_start (k_tmpl_capture)
        const std::size_t nk = static_cast<std::size_t>(idle) + 1;
        gm.g.tm_rec = env.mem.allocn<u8>(nk * kRecBytes);
        gm.g.tm_nt = env.mem.allocn<u8>(nk * 4 * kNtBytes);
        gm.g.tm_oam = env.mem.allocn<u8>(nk * 4 * kOamBytes);
        gm.g.tm_chr = gm.g.cart.chr == nullptr ? env.mem.allocn<u8>(nk * 4 * kChrRamBytes) : nullptr;
        gm.g.tm_bank = env.mem.allocn<u8>(nk * 4);
        gm.g.tm_pix = env.mem.allocn<u8>(nk * 4 * kObsPixels);
        gm.g.tm_emph = env.mem.allocn<u8>(nk * 4 * kObsH);
        gm.g.tm_meta = env.mem.allocn<RestartMeta>(nk);   // zeroed: no template taken
    }
    gm.g.tmpl_target = static_cast<u64>(kVblankDot) + static_cast<u64>(npads) * kFrameDots;
}


#define GR_BOARD_TEMPLATES(EXT, B)                                                                   \
    EXT template void launch_game<B>(const Env&, const Game&, bool, cudaStream_t, const Side&, const Range&, u32); \
    EXT template void boot_game<B>(Env&, Game&, const u8*, std::size_t, int, u32);
GR_BOARD_TEMPLATES(extern, kNrom)
GR_BOARD_TEMPLATES(extern, kUxrom)
GR_BOARD_TEMPLATES(extern, kMmc1)
GR_BOARD_TEMPLATES(extern, kMmc3)
GR_BOARD_TEMPLATES(extern, kCnrom)
GR_BOARD_TEMPLATES(extern, kMmc2)

}  // namespace gr
