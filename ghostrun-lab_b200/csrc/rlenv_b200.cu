// librlenv_b200.so: the batched NES environment for B200 behind the reference environment's C-ABI
// (rl/csrc/rlenv_api.h:8-47 and the GPU-build extras of rl/csrc/rlenv.cu:247-421). The declarations, with the
// reference interface each one replaces, are in include/rlenv_api.h.
//
// Host side: owns device memory, builds each game's cartridge view and boot / idle-frame snapshot records on the
// device, and launches the per-decision kernel sequence (envcore.cuh) on the caller's stream. Errors: int 0 ok /
// 1 failed, rlenv_create returns NULL, message in a thread-local string (rlenv_error); no C++ exception crosses
// the ABI. There is no CPU path: without a CUDA device every entry point fails with a message.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <exception>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "host.cuh"
#include "../../include/rlenv_api.h"   // the definitions below are compiled against the C-ABI declarations

using namespace gr;

namespace {

thread_local std::string g_error;
std::mutex g_specs_mu;
std::map<int, Spec> g_specs;   // rl10 game id -> reward parameters (rl10_register_game)

int fail(const std::exception& ex) { g_error = ex.what(); return 1; }

// The given launch phases of one game: main work on stream `s`, restart work on the game's side stream.
void launch_phases(Env& env, const Game& gm, bool start, cudaStream_t s, const Side& sd, const Range& rg, u32 phases) {
    switch (gm.g.cart.board) {
        case kNrom: launch_game<kNrom>(env, gm, start, s, sd, rg, phases); break;
        case kUxrom: launch_game<kUxrom>(env, gm, start, s, sd, rg, phases); break;
        case kMmc1: launch_game<kMmc1>(env, gm, start, s, sd, rg, phases); break;
        case kCnrom: launch_game<kCnrom>(env, gm, start, s, sd, rg, phases); break;
        case kMmc2: launch_game<kMmc2>(env, gm, start, s, sd, rg, phases); break;
        default: launch_game<kMmc3>(env, gm, start, s, sd, rg, phases); break;
    }
}

// The side stream of a range stepped on caller stream `s`: the game's own while level starts are on (the level
// archive and its idle chains are per game, so their kernels stay in one stream), otherwise one per caller stream.
Side range_side(Env& env, const Game& gm, cudaStream_t s) {
    if (gm.g.lv_cap > 0) return game_side(env, gm.index);
    for (const auto& c : env.range_sides)
        if (c.caller == s) return Side{c.side, c.fork, c.done};
    Env::CallerSide c{s, nullptr, nullptr, nullptr};
    ck(cudaStreamCreateWithPriority(&c.side, cudaStreamNonBlocking, env.side_priority), "range side stream");
    ck(cudaEventCreateWithFlags(&c.fork, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&c.done, cudaEventDisableTiming), "event");
    env.range_sides.push_back(c);
    return Side{c.side, c.fork, c.done};
}

// One game's decision (or a range of its envs) on stream `s`, its restart work joined back into `s`.
void launch_one(Env& env, const Game& gm, bool start, cudaStream_t s, const Range& rg) {
    const Side sd = rg.count >= 0 ? range_side(env, gm, s) : game_side(env, gm.index);
    launch_phases(env, gm, start, s, sd, rg, kPhAll);
    join_side(sd, s);
}

// Every game: a one-game env on the caller's stream; several games each on their own stream pair, concurrently,
// issued phase by phase across the games, joined back into the caller's stream.
void launch_all(Env& env, bool start, cudaStream_t s) {
    if (!env.A.actions || !env.A.masks) throw std::runtime_error("rlenv_bind was not called");
    if (env.games.size() == 1) {
        launch_one(env, env.games[0], start, s, Range{});
        return;
    }
    ck(cudaEventRecord(env.ev_begin, s), "fork");
    for (const Game& gm : env.games) ck(cudaStreamWaitEvent(env.gmain[gm.index], env.ev_begin, 0), "fork");
    for (u32 ph : {kPhFrames, kPhFinish, kPhRestart, kPhRender})
        for (const Game& gm : env.games)
            launch_phases(env, gm, start, env.gmain[gm.index], game_side(env, gm.index), Range{}, ph);
    for (const Game& gm : env.games) {
        ck(cudaEventRecord(env.gmain_done[gm.index], env.gmain[gm.index]), "join");
        ck(cudaStreamWaitEvent(s, env.gmain_done[gm.index], 0), "join");
        join_side(game_side(env, gm.index), s);
    }
}

// 4 colour numbers (6 bits) -> 3 bytes, little-endian 24-bit groups (rl/csrc/rlenv.cu:126-134 layout); 16 pixels per
// thread: one 16-byte load, three 4-byte stores.
__global__ void __launch_bounds__(256) k_pack6(const uint4* __restrict__ src, u32* __restrict__ dst, std::size_t n16) {
    for (std::size_t i = blockIdx.x * static_cast<std::size_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const uint4 q = src[i];
        auto v = [](u32 w) { return (w & 0x3Fu) | (((w >> 8) & 0x3Fu) << 6) | (((w >> 16) & 0x3Fu) << 12) | (((w >> 24) & 0x3Fu) << 18); };
        const u32 v0 = v(q.x), v1 = v(q.y), v2 = v(q.z), v3 = v(q.w);
        dst[3 * i] = v0 | (v1 << 24);
        dst[3 * i + 1] = (v1 >> 8) | (v2 << 16);
        dst[3 * i + 2] = (v2 >> 16) | (v3 << 8);
    }
}
__global__ void k_pack6_tail(const u8* src, u8* dst, std::size_t g0, std::size_t groups) {
    const std::size_t i = g0 + blockIdx.x * static_cast<std::size_t>(blockDim.x) + threadIdx.x;
    if (i >= groups) return;
    const u32 v = (src[4 * i] & 0x3Fu) | ((src[4 * i + 1] & 0x3Fu) << 6) | ((src[4 * i + 2] & 0x3Fu) << 12) | ((src[4 * i + 3] & 0x3Fu) << 18);
    dst[3 * i] = v & 0xFF; dst[3 * i + 1] = (v >> 8) & 0xFF; dst[3 * i + 2] = (v >> 16) & 0xFF;
}
__global__ void __launch_bounds__(256) k_unpack6(const u32* __restrict__ src, uint4* __restrict__ dst, std::size_t n16) {
    for (std::size_t i = blockIdx.x * static_cast<std::size_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const u32 a = src[3 * i], b = src[3 * i + 1], c = src[3 * i + 2];
        const u32 v0 = a & 0xFFFFFFu, v1 = (a >> 24) | ((b & 0xFFFFu) << 8), v2 = (b >> 16) | ((c & 0xFFu) << 16), v3 = c >> 8;
        auto w = [](u32 g) { return (g & 63u) | (((g >> 6) & 63u) << 8) | (((g >> 12) & 63u) << 16) | (((g >> 18) & 63u) << 24); };
        dst[i] = make_uint4(w(v0), w(v1), w(v2), w(v3));
    }
}
__global__ void k_unpack6_tail(const u8* src, u8* dst, std::size_t g0, std::size_t groups) {
    const std::size_t i = g0 + blockIdx.x * static_cast<std::size_t>(blockDim.x) + threadIdx.x;
    if (i >= groups) return;
    const u32 v = src[3 * i] | (static_cast<u32>(src[3 * i + 1]) << 8) | (static_cast<u32>(src[3 * i + 2]) << 16);
    dst[4 * i] = v & 63; dst[4 * i + 1] = (v >> 6) & 63; dst[4 * i + 2] = (v >> 12) & 63; dst[4 * i + 3] = (v >> 18) & 63;
}
__global__ void k_gather_rows(uint4* __restrict__ dst, const uint4* __restrict__ src, const std::int64_t* rows, std::size_t row_vecs) {
    const std::size_t j = blockIdx.x;
    const uint4* sr = src + static_cast<std::size_t>(rows[j]) * row_vecs;
    uint4* d = dst + j * row_vecs;
    for (std::size_t i = blockIdx.y * static_cast<std::size_t>(blockDim.x) + threadIdx.x; i < row_vecs; i += static_cast<std::size_t>(gridDim.y) * blockDim.x) d[i] = sr[i];
}

// One legal move per env from the masks of the last decision and 32 random bits per env: each part (d-pad 9, A 3,
// B 3, Start 2, Select 2 choices; mask bytes 0-8, 9-11, 12-14, 15-16, 17-18) uniform among its allowed choices, the
// distribution of the reference's sampler (rl/actions.py:18-20, torch.multinomial over each part's 0/1 mask), with
// the draws made by splitmix64 (Vigna's published mixer) of the env's word and the part. Packed as
// d + 9 a + 27 b + 81 start + 162 select.
__global__ void __launch_bounds__(256) k_legal_moves(const u8* __restrict__ masks, const u32* __restrict__ words,
                                                     std::int16_t* __restrict__ out, u32 n) {
    const u32 e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    const u8* m = masks + static_cast<std::size_t>(e) * 19;
    const u32 w = words[e];
    constexpr u32 kLo[5] = {0, 9, 12, 15, 17}, kCnt[5] = {9, 3, 3, 2, 2}, kMul[5] = {1, 9, 27, 81, 162};
    u32 move = 0;
#pragma unroll
    for (u32 p = 0; p < 5; ++p) {
        u32 allowed = 0;
        for (u32 c = 0; c < kCnt[p]; ++c) allowed |= (m[kLo[p] + c] ? 1u : 0u) << c;
        u64 z = ((static_cast<u64>(w) << 32) | p) + 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        const u32 k = static_cast<u32>((static_cast<u64>(static_cast<u32>(z >> 32)) * __popc(allowed)) >> 32);
        u32 pick = 0, a = allowed;   // the k-th allowed choice (0 when none is allowed)
        for (u32 j = 0; j < k; ++j) a &= a - 1;
        if (a) pick = __ffs(a) - 1;
        move += pick * kMul[p];
    }
    out[e] = static_cast<std::int16_t>(move);
}

}  // namespace

// ---- machine dump without any device allocation
//
// Who cannot allocate: a watchdog or debugger that inspects envs of a running rollout after the GPU's memory is
// spent (env state, device picture buffers and the caching allocator's pools sized to fill HBM), where the
// cudaMallocAsync staging of rlenv_dump_env fails exactly when a dump is wanted, and hosts whose memory policy fixes
// all device memory at start-up and forbids later allocation. rlenv_dump_envs_noalloc stages through the file-scope
// device array below instead and calls no cudaMalloc, cudaFree or allocating library routine.
namespace {

constexpr int kNoAllocMaxEnvs = 8;                 // RLENV_DUMP_NOALLOC_MAX_ENVS
static_assert(kNoAllocMaxEnvs == RLENV_DUMP_NOALLOC_MAX_ENVS && kDumpBytes == RLENV_DUMP_BYTES,
              "include/rlenv_api.h sizes");
constexpr int kNoAllocMaxDevices = 64;
// 8 x 23,040 B = 184,320 B. Every GPU that loads this library holds it until the process exits. Records start
// 256-byte aligned (23,040 = 90 x 256).
static __device__ __align__(256) u8 g_dump_scratch[kNoAllocMaxEnvs * kDumpBytes];
static_assert(kDumpBytes % 256 == 0, "dump records keep the scratch alignment");

std::mutex g_scratch_mu;
u8* g_scratch_ptr[kNoAllocMaxDevices] = {};        // device address of g_dump_scratch, per device, after set-up

// Set-up, once per device, with that device current: look up the array's device address and load k_dump's code
// (cudaFuncGetAttributes; with lazy loading a kernel's code is otherwise loaded at its first launch). Both can need
// device memory, so rlenv_create does this while memory is still free; a later dump then only launches and copies.
u8* noalloc_scratch(int device) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (device < 0 || device >= kNoAllocMaxDevices) throw std::runtime_error("rlenv_dump_envs_noalloc: bad device");
    if (g_scratch_ptr[device]) return g_scratch_ptr[device];
    int prev = 0;
    ck(cudaGetDevice(&prev), "rlenv_dump_envs_noalloc: cudaGetDevice");
    ck(cudaSetDevice(device), "rlenv_dump_envs_noalloc: cudaSetDevice");
    void* p = nullptr;
    cudaError_t rc = cudaGetSymbolAddress(&p, g_dump_scratch);
    cudaFuncAttributes fa{};
    if (rc == cudaSuccess) rc = cudaFuncGetAttributes(&fa, k_dump);
    const cudaError_t rc_back = cudaSetDevice(prev);
    if (rc != cudaSuccess)
        throw std::runtime_error(std::string("rlenv_dump_envs_noalloc: set-up (cudaGetSymbolAddress / cudaFuncGetAttributes) "
                                             "failed: ") + cudaGetErrorString(rc));
    if (rc_back != cudaSuccess) throw std::runtime_error("rlenv_dump_envs_noalloc: cudaSetDevice (restore) failed");
    g_scratch_ptr[device] = static_cast<u8*>(p);
    return g_scratch_ptr[device];
}

// The caller's current device for the length of a call that launches on env.device, restored on return.
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int device) {
        ck(cudaGetDevice(&prev), "cudaGetDevice");
        if (prev != device) ck(cudaSetDevice(device), "cudaSetDevice");
        else prev = -1;
    }
    ~DeviceScope() { if (prev >= 0) cudaSetDevice(prev); }
};

}  // namespace

extern "C" {

int rl10_register_game(int game_id, const double* spec, int n) {
    if (n != kSpecFields || game_id < 0) { g_error = "rl10_register_game: expected 20 fields"; return 1; }
    Spec s;
    std::memcpy(&s, spec, sizeof s);
    std::lock_guard<std::mutex> lock(g_specs_mu);
    g_specs[game_id] = s;
    return 0;
}

void* rlenv_create(int ngames, const int* game_ids, const std::uint8_t* const* roms, const std::size_t* rom_sizes,
                   const std::uint8_t* const* boot_pads, const std::size_t* boot_sizes, const int* n_envs,
                   std::uint64_t run_seed, int sticky, int idle_max, int dropout, int device) {
    Env* env = nullptr;
    try {
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
            throw std::runtime_error("no CUDA device: librlenv_b200 runs on the GPU only");
        ck(cudaSetDevice(device), "cudaSetDevice");
        env = new Env();
        env->device = device;
        int total = 0;
        for (int i = 0; i < ngames; ++i) total += n_envs[i];
        env->total = total;
        const u32 Np = static_cast<u32>((total + 1 + 31) / 32 * 32);   // + 1: boot slot
        env->Np = Np;
        std::vector<HostCart> carts;
        for (int i = 0; i < ngames; ++i) {
            carts.push_back(parse_rom(roms[i], rom_sizes[i]));
            if (carts.back().chr.empty()) env->chr_ram_any = true;
        }
        DevMem& M = env->mem;
        env->A.st = alloc_state_view(M, Np, env->chr_ram_any, true);
        EnvArgs& A = env->A;
        const std::size_t N = static_cast<std::size_t>(total) + 1;
        A.trk = M.allocn<Tracker>(N, true);
        A.drop = M.allocn<Dropout>(N, true);
        A.target = M.allocn<u64>(N, true);
        A.ep_frame = M.allocn<u32>(N, true);
        A.prev_applied = M.allocn<int16_t>(N, true);
        A.sticky_seed = M.allocn<u64>(N, true);
        A.sticky_ctr = M.allocn<u64>(N, true);
        A.episode = M.allocn<u32>(N, true);
        A.ep_ret = M.allocn<float>(N, true);
        A.ep_len = M.allocn<i32>(N, true);
        A.ep_maxlvl = M.allocn<i32>(N, true);
        A.ep_idle = M.allocn<i32>(N, true);
        A.fault = M.allocn<u32>(N, true);
        A.resetting = M.allocn<u8>(N);
        A.render_seq = M.allocn<u8>(static_cast<std::size_t>(N) * kFramesPerDecision);   // transient: not saved
        A.render_stats = M.allocn<unsigned long long>(2);   // transient: not saved
        A.tm_used = M.allocn<u8>(N);
        A.list = M.allocn<u32>(N);                                    // per game: its slice [game_e0, game_e0 + n)
        A.list_count = M.allocn<u32>(static_cast<std::size_t>(ngames) + 1 + N);   // per game, then per range start
        {
            std::vector<u32> init(N, 0xFFFFFFFFu);
            ck(cudaMemcpy(A.episode, init.data(), N * 4, cudaMemcpyHostToDevice), "episode init");
        }
        A.run_seed = run_seed;
        A.sticky = sticky;
        A.idle_max = idle_max;
        A.dropout = dropout;
        A.no_render = 0;
        A.episode_level_end = -1;
        int offset = 0;
        for (int i = 0; i < ngames; ++i) {
            Game gm;
            gm.game_id = game_ids[i];
            gm.index = i;
            {
                std::lock_guard<std::mutex> lock(g_specs_mu);
                auto it = g_specs.find(game_ids[i]);
                if (it == g_specs.end())
                    throw std::runtime_error("game id " + std::to_string(game_ids[i]) + " has no reward spec (rl10_register_game)");
                if (it->second.reader != 1.0)
                    throw std::runtime_error("game id " + std::to_string(game_ids[i]) + ": only the synthetic RAM reader is built");
                gm.g.spec = it->second;
            }
            const HostCart& hc = carts[i];
            CartView& C = gm.g.cart;
            u8* prg = M.allocn<u8>(hc.prg.size());
            ck(cudaMemcpy(prg, hc.prg.data(), hc.prg.size(), cudaMemcpyHostToDevice), "prg");
            C.prg = prg;
            // NROM / CNROM read the staged window through this mask: the whole 16 / 32 KB image (a 16 KB one
            // mirrored); CNROM maps pages 0-3 of a larger image, its first 32 KB
            C.prg_mask = static_cast<u32>(std::min<std::size_t>(hc.prg.size(), 32768) - 1);
            if (!hc.chr.empty()) {
                u8* chr = M.allocn<u8>(hc.chr.size());
                ck(cudaMemcpy(chr, hc.chr.data(), hc.chr.size(), cudaMemcpyHostToDevice), "chr");
                C.chr = chr;
                C.chr_size = static_cast<u32>(hc.chr.size());
                const std::vector<u32> x = expand_chr(hc.chr);
                u32* cx = M.allocn<u32>(x.size());
                ck(cudaMemcpy(cx, x.data(), x.size() * 4, cudaMemcpyHostToDevice), "chrx");
                C.chrx = cx;
                C.chr_tiles = 512;
                gm.chrx_smem = hc.board == kNrom || hc.board == kUxrom;
            } else {
                C.chr = nullptr;
                C.chr_size = 0;
                C.chrx = nullptr;
            }
            C.board = hc.board;
            // PRG staged in the emulation blocks' shared memory: the whole mapped window on NROM / CNROM (the first
            // 16 / 32 KB), else the last 16 KB
            const bool fixed = hc.board == kNrom || hc.board == kCnrom;
            C.prg_stage_bytes = fixed ? C.prg_mask + 1u : std::min<u32>(16384u, static_cast<u32>(hc.prg.size()));
            C.prg_stage_base = fixed ? 0u : static_cast<u32>(hc.prg.size()) - C.prg_stage_bytes;
            C.arrangement = hc.arrangement;
            C.bank_mask = hc.bank_mask;
            C.fixed_base = hc.fixed_base;
            C.prg_page_mask = hc.prg_page_mask;
            C.chr_page_mask = hc.chr_page_mask;
            gm.g.e0 = static_cast<u32>(offset);
            gm.g.game_e0 = static_cast<u32>(offset);
            gm.g.n = static_cast<u32>(n_envs[i]);
            gm.g.start_ok = gm.g.spec.start_ok != 0.0;
            gm.g.select_ok = gm.g.spec.select_ok != 0.0;
            offset += n_envs[i];
            const u32 boot_slot = static_cast<u32>(total);
            switch (hc.board) {
                case kNrom: boot_game<kNrom>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
                case kUxrom: boot_game<kUxrom>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
                case kMmc1: boot_game<kMmc1>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
                case kCnrom: boot_game<kCnrom>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
                case kMmc2: boot_game<kMmc2>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
                default: boot_game<kMmc3>(*env, gm, boot_pads[i], boot_sizes[i], idle_max, boot_slot); break;
            }
            env->games.push_back(gm);
        }
        ck(cudaEventCreateWithFlags(&env->ev, cudaEventDisableTiming), "event");
        ck(cudaEventCreateWithFlags(&env->ev_begin, cudaEventDisableTiming), "event");
        int least = 0, greatest = 0;
        ck(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
        env->side_priority = greatest;
        for (std::size_t gi = 0; gi < env->games.size(); ++gi) {
            cudaStream_t q = nullptr;
            cudaEvent_t e = nullptr;
            ck(cudaStreamCreateWithPriority(&q, cudaStreamNonBlocking, least), "game stream");
            env->gmain.push_back(q);
            ck(cudaStreamCreateWithPriority(&q, cudaStreamNonBlocking, greatest), "side stream");
            env->gside.push_back(q);
            ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
            env->gfork.push_back(e);
            ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
            env->gmain_done.push_back(e);
            ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
            env->gside_done.push_back(e);
        }
        env->timer = new KTimer();
        noalloc_scratch(device);   // rlenv_dump_envs_noalloc's per-device set-up, while device memory is still free
        ck(cudaDeviceSynchronize(), "create");
        return env;
    } catch (const std::exception& ex) {
        g_error = ex.what();
        delete env;
        return nullptr;
    }
}

int rlenv_num_envs(void* h) { return static_cast<Env*>(h)->total; }
int rlenv_num_games(void* h) { return static_cast<int>(static_cast<Env*>(h)->games.size()); }
void rlenv_set_episode_level_end(void* h, int level) { static_cast<Env*>(h)->A.episode_level_end = level; }
void rlenv_set_no_render(void* h, int v) { static_cast<Env*>(h)->A.no_render = v; }

void rlenv_bind(void* h, const std::int16_t* actions, std::uint8_t* obs, std::uint8_t* emph, float* reward,
                std::uint8_t* done, std::uint8_t* masks, std::uint8_t* timeline, std::uint8_t* pads,
                std::uint32_t* events, float* info) {
    EnvArgs& A = static_cast<Env*>(h)->A;
    A.actions = actions; A.obs = obs; A.emph = emph; A.reward = reward; A.done = done; A.masks = masks;
    A.timeline = timeline; A.pads = pads; A.events = events; A.info = info;
}
void rlenv_bind_parts(void* h, float* parts) { static_cast<Env*>(h)->A.parts = parts; }
// Pictures as packed 6-bit colour numbers [N, 4, 224, 180] (the rl_pack6 layout of obs) written by the renderer
// itself instead of the [N, 4, 224, 240] bytes; nullptr restores the byte output.
void rlenv_bind_obs_pack6(void* h, std::uint8_t* packed) { static_cast<Env*>(h)->A.packed = packed; }
void rlenv_bind_obs(void* h, std::uint8_t* obs, std::uint8_t* emph) {
    EnvArgs& A = static_cast<Env*>(h)->A;
    A.obs = obs;
    A.emph = emph;
}

int rlenv_start(void* h, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        auto s = static_cast<cudaStream_t>(stream);
        launch_all(env, true, s);
        if (!env.A.no_render) {   // every env just made a boot (or level) restart: take the restart templates
            for (const Game& gm : env.games) {
                k_tmpl_capture<<<gm.g.idle_tmpl + 1, 128, 0, s>>>(gm.g, env.A);
                check_launch("k_tmpl_capture");
            }
        }
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rlenv_step(void* h, void* stream) {
    try {
        launch_all(*static_cast<Env*>(h), false, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

std::size_t rlenv_state_bytes(void* h) {
    std::size_t n = 0;
    for (const auto& pb : static_cast<Env*>(h)->mem.state) n += pb.second;
    return n;
}
int rlenv_save(void* h, std::uint8_t* out, void* stream) {
    try {
        auto s = static_cast<cudaStream_t>(stream);
        for (const auto& pb : static_cast<Env*>(h)->mem.state) {
            ck(cudaMemcpyAsync(out, pb.first, pb.second, cudaMemcpyDeviceToHost, s), "save");
            out += pb.second;
        }
        ck(cudaStreamSynchronize(s), "save");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rlenv_load(void* h, const std::uint8_t* in, void* stream) {
    try {
        auto s = static_cast<cudaStream_t>(stream);
        Env& env = *static_cast<Env*>(h);
        for (const auto& pb : env.mem.state) {
            ck(cudaMemcpyAsync(pb.first, in, pb.second, cudaMemcpyHostToDevice, s), "load");
            in += pb.second;
        }
        for (const Game& gm : env.games)   // level-start slots may have changed: their idle chains are remade
            if (gm.g.lv_chain_ok) ck(cudaMemsetAsync(gm.g.lv_chain_ok, 0, static_cast<std::size_t>(gm.g.lv_cap) * 4, s), "load");
        ck(cudaStreamSynchronize(s), "load");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

const char* rlenv_error() { return g_error.c_str(); }
void rlenv_destroy(void* h) { delete static_cast<Env*>(h); }

// ---- level starts and places (rl/csrc/rlenv.cu:331-362, rl/csrc/rlenv_build.hpp:212-252)
// Room for `cap` saved states per game, empty; slots < `levels` are level entrances saved by the archive after each
// decision, the rest places saved by rlenv_place_save. Call once, before start / load. The new state (episode start
// slots, then per game: records, trackers, frame targets, frames, deaths) is saved after everything else, so a state
// saved without level starts is a prefix of one saved with them.
int rlenv_enable_places(void* h, int cap, int levels) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (env.lv_cap != 0 || cap <= 0 || levels <= 0 || levels > cap)
            throw std::logic_error("level starts: enable once, 0 < levels <= cap");
        DevMem& M = env.mem;
        const std::size_t N = static_cast<std::size_t>(env.total) + 1;
        env.A.ep_start = M.allocn<i32>(N, true);
        env.A.lv_chained = M.allocn<u8>(N);
        {
            std::vector<i32> none(N, -1);
            ck(cudaMemcpy(env.A.ep_start, none.data(), N * 4, cudaMemcpyHostToDevice), "level starts");
        }
        const std::size_t C = static_cast<std::size_t>(cap);
        for (Game& gm : env.games) {
            GameArgs& g = gm.g;
            g.lv_cap = static_cast<u32>(cap);
            g.lv_levels = static_cast<u32>(levels);
            g.lv_rec = M.allocn<u8>(C * kRecBytes, true);
            g.lv_st = M.allocn<Tracker>(C, true);
            g.lv_target = M.allocn<u64>(C, true);
            g.lv_frame = M.allocn<u32>(C, true);
            g.lv_deaths = M.allocn<i32>(C, true);
            g.lv_claim = M.allocn<unsigned long long>(C);
            u32* cdf = M.allocn<u32>(C);
            g.lv_cdf = cdf;
            std::vector<i32> none(C, -1);
            ck(cudaMemcpy(g.lv_deaths, none.data(), C * 4, cudaMemcpyHostToDevice), "level starts");
            std::vector<unsigned long long> free_(C, ~0ull);
            ck(cudaMemcpy(g.lv_claim, free_.data(), C * 8, cudaMemcpyHostToDevice), "level starts");
            // idle chains (derived data, not saved): records after 1..idle_max idle frames of each slot
            g.lv_idle_n = env.A.idle_max > 0 ? static_cast<u32>(env.A.idle_max) : 0u;
            g.lv_chain_ok = M.allocn<u32>(C);
            if (g.lv_idle_n > 0) {
                g.lv_idle_rec = M.allocn<u8>(C * g.lv_idle_n * kRecBytes);
                g.lv_idle_fault = M.allocn<u32>(C * g.lv_idle_n);
                g.lv_scratch = alloc_state_view(M, static_cast<u32>((C + 31) / 32 * 32), g.cart.chr == nullptr, false);
            }
        }
        env.lv_cap = cap;
        env.lv_levels = levels;
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rlenv_enable_level_starts(void* h, int cap) { return rlenv_enable_places(h, cap, cap); }

// Level-start share p and level weights (cdf: lv_cap u32 in host memory, nullptr = uniform over the saved slots)
// of game gi, for episodes that start from the next launch on. Synchronous.
void rlenv_set_level_plan(void* h, int gi, double p, const std::uint32_t* cdf) {
    Env& env = *static_cast<Env*>(h);
    if (gi < 0 || gi >= static_cast<int>(env.games.size())) return;
    GameArgs& g = env.games[static_cast<std::size_t>(gi)].g;
    if (g.lv_cap == 0) return;
    g.lv_thresh = static_cast<u32>(p <= 0.0 ? 0.0 : p >= 1.0 ? 4294967295.0 : p * 4294967296.0);
    g.lv_weighted = cdf != nullptr ? 1u : 0u;
    if (cdf) {
        const cudaError_t e = cudaMemcpy(const_cast<u32*>(g.lv_cdf), cdf, static_cast<std::size_t>(g.lv_cap) * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) g_error = std::string("set_level_plan: ") + cudaGetErrorString(e);
    }
}
void rlenv_bind_start(void* h, std::int32_t* start_out) { static_cast<Env*>(h)->A.start_out = start_out; }
void rlenv_bind_level(void* h, std::int32_t* level_out) { static_cast<Env*>(h)->A.level_out = level_out; }
void rlenv_bind_progress(void* h, float* progress_out) { static_cast<Env*>(h)->A.progress_out = progress_out; }

// Deaths of each saved slot of game gi (-1 = nothing saved), lv_cap entries into host memory (synchronous).
int rlenv_level_deaths(void* h, int gi, std::int32_t* out, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (gi < 0 || gi >= static_cast<int>(env.games.size())) throw std::runtime_error("level_deaths: bad game");
        const GameArgs& g = env.games[static_cast<std::size_t>(gi)].g;
        if (g.lv_cap == 0) return 0;
        auto s = static_cast<cudaStream_t>(stream);
        ck(cudaMemcpyAsync(out, g.lv_deaths, static_cast<std::size_t>(g.lv_cap) * 4, cudaMemcpyDeviceToHost, s), "level_deaths");
        ck(cudaStreamSynchronize(s), "level_deaths");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// env_idx[j] (index within game gi) -> place slot slot_idx[j] (device int32 arrays; slots < levels are skipped),
// on `stream` after the step.
int rlenv_place_save(void* h, int gi, const std::int32_t* env_idx, const std::int32_t* slot_idx, int count, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (gi < 0 || gi >= static_cast<int>(env.games.size())) throw std::runtime_error("place_save: bad game");
        const GameArgs& g = env.games[static_cast<std::size_t>(gi)].g;
        if (g.lv_cap == 0 || count <= 0) return 0;
        k_place_save<<<count, 128, 0, static_cast<cudaStream_t>(stream)>>>(g, env.A, env_idx, slot_idx);
        check_launch("k_place_save");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// Slot src[j] -> slot dst[j] of game gi, whole saved state (host int32 arrays; synchronous).
int rlenv_place_copy(void* h, int gi, const std::int32_t* src, const std::int32_t* dst, int count, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (gi < 0 || gi >= static_cast<int>(env.games.size())) throw std::runtime_error("place_copy: bad game");
        const GameArgs& g = env.games[static_cast<std::size_t>(gi)].g;
        const int cap = static_cast<int>(g.lv_cap);
        for (int i = 0; i < count; ++i)
            if (src[i] < 0 || dst[i] < 0 || src[i] >= cap || dst[i] >= cap) throw std::runtime_error("place_copy: bad slot");
        auto s = static_cast<cudaStream_t>(stream);
        for (int i = 0; i < count; ++i) {
            const std::size_t a = static_cast<std::size_t>(src[i]), b = static_cast<std::size_t>(dst[i]);
            if (g.lv_chain_ok) ck(cudaMemsetAsync(g.lv_chain_ok + b, 0, 4, s), "place_copy");   // remade next decision
            ck(cudaMemcpyAsync(g.lv_rec + b * kRecBytes, g.lv_rec + a * kRecBytes, kRecBytes, cudaMemcpyDeviceToDevice, s), "place_copy");
            ck(cudaMemcpyAsync(g.lv_st + b, g.lv_st + a, sizeof(Tracker), cudaMemcpyDeviceToDevice, s), "place_copy");
            ck(cudaMemcpyAsync(g.lv_target + b, g.lv_target + a, 8, cudaMemcpyDeviceToDevice, s), "place_copy");
            ck(cudaMemcpyAsync(g.lv_frame + b, g.lv_frame + a, 4, cudaMemcpyDeviceToDevice, s), "place_copy");
            ck(cudaMemcpyAsync(g.lv_deaths + b, g.lv_deaths + a, 4, cudaMemcpyDeviceToDevice, s), "place_copy");
        }
        ck(cudaStreamSynchronize(s), "place_copy");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// Sizes of one game's saved-slot state, as rl/csrc/rlenv.cu:356-360: stride of a slot's state record, key slots
// (none: the synthetic reader keeps no key set), tracker bytes, cap, levels.
void rlenv_level_layout(void* h, int gi, std::uint32_t* out) {
    const Env& env = *static_cast<Env*>(h);
    const GameArgs& g = env.games[static_cast<std::size_t>(gi)].g;
    out[0] = static_cast<u32>(kRecBytes);
    out[1] = 0;
    out[2] = static_cast<u32>(sizeof(Tracker));
    out[3] = g.lv_cap;
    out[4] = g.lv_levels;
}

int rlenv_step_game(void* h, int gi, std::uint8_t* obs, std::uint8_t* emph, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (gi < 0 || gi >= static_cast<int>(env.games.size())) throw std::runtime_error("step_game: bad game index");
        auto s = static_cast<cudaStream_t>(stream);
        Range rg;
        rg.obs = obs; rg.emph = emph;
        launch_one(env, env.games[gi], false, s, rg);
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rlenv_step_range(void* h, int gi, int start, int count, std::uint8_t* obs, std::uint8_t* emph, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (gi < 0 || gi >= static_cast<int>(env.games.size())) throw std::runtime_error("step_range: bad game index");
        const Game& gm = env.games[gi];
        if (start < 0 || count <= 0 || start + count > static_cast<int>(gm.g.n)) throw std::runtime_error("step_range: bad range");
        auto s = static_cast<cudaStream_t>(stream);
        Range rg;
        rg.start = start; rg.count = count; rg.obs = obs; rg.emph = emph;
        launch_one(env, gm, false, s, rg);
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// ---- host-memory rollout storage and the 6-bit picture format (rl/csrc/rlenv.cu:369-421)
void* rl_host_alloc(std::size_t bytes) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) { g_error = "cudaHostAlloc failed"; return nullptr; }
    return p;
}
void rl_host_free(void* p) { cudaFreeHost(p); }
int rl_pack6(const void* src, void* dst, std::size_t pixels, void* stream) {
    try {
        if (pixels % 4) throw std::runtime_error("pack6: pixel count must be divisible by four");
        auto s = static_cast<cudaStream_t>(stream);
        const std::size_t groups = pixels / 4;
        const bool vec = (reinterpret_cast<std::uintptr_t>(src) % 16 == 0) && (reinterpret_cast<std::uintptr_t>(dst) % 4 == 0);
        const std::size_t n16 = vec ? pixels / 16 : 0;
        if (n16) {
            const unsigned blocks = static_cast<unsigned>(std::min<std::size_t>((n16 + 255) / 256, 148 * 32));
            k_pack6<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(src), static_cast<u32*>(dst), n16);
        }
        const std::size_t g0 = n16 * 4;
        if (groups > g0)
            k_pack6_tail<<<static_cast<unsigned>((groups - g0 + 255) / 256), 256, 0, s>>>(static_cast<const u8*>(src), static_cast<u8*>(dst), g0, groups);
        check_launch("pack6");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rl_unpack6(const void* src, void* dst, std::size_t pixels, void* stream) {
    try {
        if (pixels % 4) throw std::runtime_error("unpack6: pixel count must be divisible by four");
        auto s = static_cast<cudaStream_t>(stream);
        const std::size_t groups = pixels / 4;
        const bool vec = (reinterpret_cast<std::uintptr_t>(src) % 4 == 0) && (reinterpret_cast<std::uintptr_t>(dst) % 16 == 0);
        const std::size_t n16 = vec ? pixels / 16 : 0;
        if (n16) {
            const unsigned blocks = static_cast<unsigned>(std::min<std::size_t>((n16 + 255) / 256, 148 * 32));
            k_unpack6<<<blocks, 256, 0, s>>>(static_cast<const u32*>(src), static_cast<uint4*>(dst), n16);
        }
        const std::size_t g0 = n16 * 4;
        if (groups > g0)
            k_unpack6_tail<<<static_cast<unsigned>((groups - g0 + 255) / 256), 256, 0, s>>>(static_cast<const u8*>(src), static_cast<u8*>(dst), g0, groups);
        check_launch("unpack6");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
int rl_memcpy_async(void* dst, const void* src, std::size_t bytes, void* stream) {
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        g_error = std::string("memcpy: ") + cudaGetErrorString(cudaGetLastError());
        return 1;
    }
    return 0;
}
int rl_gather_rows(void* dst, const void* src, const std::int64_t* rows, int nrows, std::size_t row_bytes, void* stream) {
    try {
        if (row_bytes % 16) throw std::runtime_error("gather_rows: row_bytes must be a multiple of 16");
        if (nrows <= 0) return 0;
        dim3 grid(static_cast<unsigned>(nrows), 32);
        k_gather_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), rows, row_bytes / 16);
        check_launch("gather_rows");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}
// Copy-engine gather: dst[t * n + j] = src[t * N + envs[j]] for t < T (one 2-D copy per env; envs in host memory).
int rl_gather_envs(void* dst, const void* src, const std::int64_t* envs, int n, int T, int N, std::size_t row_bytes, void* stream) {
    auto s = static_cast<cudaStream_t>(stream);
    for (int j = 0; j < n; ++j) {
        if (cudaMemcpy2DAsync(static_cast<char*>(dst) + j * row_bytes, static_cast<std::size_t>(n) * row_bytes,
                              static_cast<const char*>(src) + envs[j] * row_bytes, static_cast<std::size_t>(N) * row_bytes,
                              row_bytes, static_cast<std::size_t>(T), cudaMemcpyDefault, s) != cudaSuccess) {
            g_error = "gather2d failed";
            return 1;
        }
    }
    return 0;
}

// One legal move per env (see k_legal_moves): masks u8[n,19] (the env's masks output), words u32[n] random bits,
// actions i16[n]; device pointers, asynchronous on `stream`.
int rl_legal_moves(const void* masks, const void* words, void* actions, int n, void* stream) {
    try {
        if (n < 0 || (n > 0 && (!masks || !words || !actions))) throw std::runtime_error("rl_legal_moves: bad arguments");
        if (n == 0) return 0;
        k_legal_moves<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const u8*>(masks), static_cast<const u32*>(words), static_cast<std::int16_t*>(actions),
            static_cast<u32>(n));
        check_launch("k_legal_moves");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// ---- measurement: per-kernel device time on the launching stream (CUDA events), launch counts
void rlenv_set_timing(void* h, int on) {
    KTimer& T = *static_cast<Env*>(h)->timer;
    T.collect();
    T.on = on != 0;
}
void rlenv_bind_episode_counters(void* h, double* acc) { static_cast<Env*>(h)->A.ep_acc = acc; }
void rlenv_set_timing_kinds(void* h, unsigned mask) {
    KTimer& T = *static_cast<Env*>(h)->timer;
    T.collect();
    T.mask = mask;
}
// out[0..5] = ms of frames / render / finish / restart frames / restart render / pack6 kernels since the last reset,
// out[6..11] their launch counts, out[12] all launches; reset != 0 clears the counters afterwards.
int rlenv_timing(void* h, double* out, int reset) {
    try {
        KTimer& T = *static_cast<Env*>(h)->timer;
        T.collect();
        for (int k = 0; k < kKinds; ++k) { out[k] = T.ms[k]; out[kKinds + k] = static_cast<double>(T.launches[k]); }
        out[2 * kKinds] = static_cast<double>(T.total_launches);
        if (reset) T.reset();
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// Canonical machine state of global env `ge` into host memory (layout: include/rlenv_api.h).
std::size_t rlenv_dump_bytes() { return kDumpBytes; }
int rlenv_dump_env(void* h, int ge, std::uint8_t* host_out, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (ge < 0 || ge >= env.total) throw std::runtime_error("dump: bad env index");
        DeviceScope on(env.device);
        auto s = static_cast<cudaStream_t>(stream);
        u8* d = nullptr;
        ck(cudaMallocAsync(reinterpret_cast<void**>(&d), kDumpBytes, s), "dump alloc");
        k_dump<<<1, 32, 0, s>>>(env.A.st, static_cast<u32>(ge), env.chr_ram_any ? 1u : 0u, d);
        check_launch("k_dump");
        ck(cudaMemcpyAsync(host_out, d, kDumpBytes, cudaMemcpyDeviceToHost, s), "dump copy");
        ck(cudaFreeAsync(d, s), "dump free");
        ck(cudaStreamSynchronize(s), "dump");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// How the pictures since the last reset were drawn: out[0] frames drawn by the sequential renderer (k_render_seq),
// out[1] lines with a write inside their drawn part drawn exactly by the walk (host memory, synchronous).
int rlenv_render_stats(void* h, std::uint64_t* out, int reset, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (!out) throw std::runtime_error("rlenv_render_stats: null pointer");
        auto s = static_cast<cudaStream_t>(stream);
        unsigned long long v[2] = {0, 0};
        ck(cudaMemcpyAsync(v, env.A.render_stats, sizeof v, cudaMemcpyDeviceToHost, s), "render stats");
        if (reset) ck(cudaMemsetAsync(env.A.render_stats, 0, sizeof v, s), "render stats reset");
        ck(cudaStreamSynchronize(s), "render stats");
        out[0] = v[0]; out[1] = v[1];
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// Per-env RL scalars of global env ge: target, ep_frame, episode, fault, sticky_ctr (host memory, synchronous).
int rlenv_env_scalars(void* h, int ge, std::uint64_t* out, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        auto s = static_cast<cudaStream_t>(stream);
        u64 t = 0, sc = 0;
        u32 f = 0, ep = 0, fl = 0;
        ck(cudaMemcpyAsync(&t, env.A.target + ge, 8, cudaMemcpyDeviceToHost, s), "scalars");
        ck(cudaMemcpyAsync(&f, env.A.ep_frame + ge, 4, cudaMemcpyDeviceToHost, s), "scalars");
        ck(cudaMemcpyAsync(&ep, env.A.episode + ge, 4, cudaMemcpyDeviceToHost, s), "scalars");
        ck(cudaMemcpyAsync(&fl, env.A.fault + ge, 4, cudaMemcpyDeviceToHost, s), "scalars");
        ck(cudaMemcpyAsync(&sc, env.A.sticky_ctr + ge, 8, cudaMemcpyDeviceToHost, s), "scalars");
        ck(cudaStreamSynchronize(s), "scalars");
        out[0] = t; out[1] = f; out[2] = ep; out[3] = fl; out[4] = sc;
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

// rlenv_dump_env for envs[0..n) in one call, n <= 8, without allocating: n x 23,040 bytes into host_out, same
// layout. k_dump zero-fills each record it writes before setting the fields, so nothing of an earlier call's
// contents (the array keeps them) reaches the output. Every call and every handle on a device shares the one array:
// calls whose work overlaps on the GPU (two host threads, or two streams) race. A call runs its kernels and copy on
// `stream` and synchronises it before returning.
int rlenv_dump_envs_noalloc(void* h, const int* envs, int n, std::uint8_t* host_out, void* stream) {
    try {
        Env& env = *static_cast<Env*>(h);
        if (n < 1 || n > kNoAllocMaxEnvs)
            throw std::runtime_error("rlenv_dump_envs_noalloc: " + std::to_string(n) + " envs requested; one call dumps 1.." +
                                     std::to_string(kNoAllocMaxEnvs) + " envs (fixed scratch of " +
                                     std::to_string(kNoAllocMaxEnvs) + " x RLENV_DUMP_BYTES)");
        if (!envs || !host_out) throw std::runtime_error("rlenv_dump_envs_noalloc: null pointer");
        for (int i = 0; i < n; ++i)
            if (envs[i] < 0 || envs[i] >= env.total) throw std::runtime_error("rlenv_dump_envs_noalloc: bad env index");
        DeviceScope on(env.device);
        u8* scratch = noalloc_scratch(env.device);   // looked up by rlenv_create already
        auto s = static_cast<cudaStream_t>(stream);
        for (int i = 0; i < n; ++i) {
            k_dump<<<1, 32, 0, s>>>(env.A.st, static_cast<u32>(envs[i]), env.chr_ram_any ? 1u : 0u,
                                    scratch + static_cast<std::size_t>(i) * kDumpBytes);
            check_launch("k_dump");
        }
        ck(cudaMemcpyAsync(host_out, scratch, static_cast<std::size_t>(n) * kDumpBytes, cudaMemcpyDeviceToHost, s),
           "rlenv_dump_envs_noalloc: copy");
        ck(cudaStreamSynchronize(s), "rlenv_dump_envs_noalloc");
        return 0;
    } catch (const std::exception& ex) { return fail(ex); }
}

}  // extern "C"
