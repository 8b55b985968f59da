// C-ABI of librlenv_b200.so, the batched NES environment for B200 (ghostrun-lab_b200/csrc). Every entry point the
// reference's Python side binds (rl/rlenv.py:76-119 _load) is here with the same name, argument meaning and error
// behaviour; each line cites the reference declaration it replaces. Plain pointers and sizes only: all buffers given
// to rlenv_bind* are device pointers, `stream` is a cudaStream_t (the caller's torch stream). Calls return int 0 on
// success and non-zero on failure with a message in rlenv_error() (thread-local); rlenv_create returns NULL on
// failure; no C++ exception crosses the ABI. There is no CPU path: without a CUDA device every call fails.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ---------------------------------------------------------------- lifecycle (rl/csrc/rlenv_api.h:9-12, 43-46)

// rl/csrc/rlenv_api.h:9-11. game_ids: rl10 game ids (0..11 the reference's commercial games, 12..25 the seeded
// synthetic games of ghostrun-lab_b200/synth.py; a game needs its reward spec registered first, rl10_register_game).
// roms: iNES images (mappers 0 NROM, 1 MMC1, 2 UxROM, 3 CNROM, 4 MMC3, 9 MMC2); boot_pads: pad byte of every frame from power-on to
// the boot snapshot; n_envs: envs per game. sticky / dropout: 0/1; idle_max: 0..idle_max random idle frames at
// episode starts; device: CUDA device index.
void* rlenv_create(int ngames, const int* game_ids, const uint8_t* const* roms, const size_t* rom_sizes,
                   const uint8_t* const* boot_pads, const size_t* boot_sizes, const int* n_envs, uint64_t run_seed,
                   int sticky, int idle_max, int dropout, int device);
int rlenv_num_envs(void* h);                                              // rl/csrc/rlenv_api.h:12
const char* rlenv_error(void);                                            // rl/csrc/rlenv_api.h:45
void rlenv_destroy(void* h);                                              // rl/csrc/rlenv_api.h:46

// ---------------------------------------------------------------- outputs (rl/csrc/rlenv_api.h:15-21)

// rl/csrc/rlenv_api.h:15-17: actions i16[N]; obs u8[N,4,224,240]; emph u8[N,4,224]; reward f32[N]; done u8[N];
// masks u8[N,19]; timeline u8[N,8,45]; pads u8[N,4]; events u32[N]; info f32[N,8]. Takes effect at the next call.
void rlenv_bind(void* h, const int16_t* actions, uint8_t* obs, uint8_t* emph, float* reward, uint8_t* done,
                uint8_t* masks, uint8_t* timeline, uint8_t* pads, uint32_t* events, float* info);
void rlenv_bind_parts(void* h, float* parts);                             // rl/csrc/rlenv_api.h:19, f32[N,7]
void rlenv_bind_obs(void* h, uint8_t* obs, uint8_t* emph);                // rl/csrc/rlenv_api.h:21
// Extension (no reference counterpart; replaces the reference's rl_pack6 pass after the step, rl/csrc/rlenv.cu:
// 380-386, when set): the renderer writes the pictures directly as packed 6-bit colour numbers u8[N,4,224,180] in
// the rl_pack6 layout; NULL restores the byte output.
void rlenv_bind_obs_pack6(void* h, uint8_t* packed);

// ---------------------------------------------------------------- level starts and places (rl/csrc/rlenv_api.h:22-39)

// rl/csrc/rlenv_api.h:26,36: room for `cap` saved states per game (call once, before start / load); slots < levels
// are level entrances saved after each decision by the best arrival (fewest deaths, then lowest env), the rest
// places. enable_level_starts(h, cap) = enable_places(h, cap, cap). The state they add is saved last (a state
// saved without them is a prefix).
int rlenv_enable_level_starts(void* h, int cap);                          // rl/csrc/rlenv_api.h:26
int rlenv_enable_places(void* h, int cap, int levels);                    // rl/csrc/rlenv_api.h:36
// rl/csrc/rlenv_api.h:27: chance p that a new episode of game gi starts from a saved slot, and cumulative slot
// weights * 2^32 (cap entries in host memory; NULL = uniform over the saved slots). Between decisions.
void rlenv_set_level_plan(void* h, int gi, double p, const uint32_t* cdf);
void rlenv_bind_start(void* h, int32_t* start_out);      // rl/csrc/rlenv_api.h:28: [N] start slot of a finished episode, -1 power-on
void rlenv_bind_level(void* h, int32_t* level_out);      // rl/csrc/rlenv_api.h:29: [N] level after each decision, -1 unknown
void rlenv_bind_progress(void* h, float* progress_out);  // rl/csrc/rlenv_api.h:30: [N] progress / progress_unit, NaN invalid
int rlenv_level_deaths(void* h, int gi, int32_t* host_out, void* stream);  // rl/csrc/rlenv_api.h:31 (synchronous)
// rl/csrc/rlenv_api.h:37: env_idx[j] (index within game gi) -> slot_idx[j] (skipped unless levels <= slot < cap);
// device int32 arrays, after a step on the same stream.
int rlenv_place_save(void* h, int gi, const int32_t* env_idx, const int32_t* slot_idx, int count, void* stream);
// rl/csrc/rlenv_api.h:38: slot src[j] -> dst[j] of game gi, host int32 arrays, synchronous.
int rlenv_place_copy(void* h, int gi, const int32_t* src, const int32_t* dst, int count, void* stream);
// rl/csrc/rlenv_api.h:39: out[5] = slot stride, key slots (0: the synthetic reader keeps no key set), tracker
// bytes, cap, levels.
void rlenv_level_layout(void* h, int gi, uint32_t* out);

// ---------------------------------------------------------------- decisions (rl/csrc/rlenv_api.h:40-41)

int rlenv_start(void* h, void* stream);   // rl/csrc/rlenv_api.h:40: first episode of every env
int rlenv_step(void* h, void* stream);    // rl/csrc/rlenv_api.h:41: one decision (4 frames) of every env
int rlenv_num_games(void* h);                                             // rl/csrc/rlenv.cu:247
int rlenv_step_game(void* h, int gi, uint8_t* obs, uint8_t* emph, void* stream);               // rl/csrc/rlenv.cu:248-255
int rlenv_step_range(void* h, int gi, int start, int count, uint8_t* obs, uint8_t* emph, void* stream);  // rl/csrc/rlenv.cu:257-267
void rlenv_set_episode_level_end(void* h, int level);                     // rl/csrc/rlenv_api.h:14
void rlenv_set_no_render(void* h, int v);                                 // rl/csrc/rlenv.cu:364-366

// ---------------------------------------------------------------- exact resume (rl/csrc/rlenv_api.h:42-44)

size_t rlenv_state_bytes(void* h);                                        // rl/csrc/rlenv_api.h:42
int rlenv_save(void* h, uint8_t* host_out, void* stream);                 // rl/csrc/rlenv_api.h:43 (synchronous)
int rlenv_load(void* h, const uint8_t* host_in, void* stream);            // rl/csrc/rlenv_api.h:44 (synchronous)

// ---------------------------------------------------------------- 6-bit pictures and host storage (rl/csrc/rlenv.cu:369-421)

void* rl_host_alloc(size_t bytes);                                        // rl/csrc/rlenv.cu:371-378 (pinned, portable)
void rl_host_free(void* p);                                               // rl/csrc/rlenv.cu:379
int rl_pack6(const void* src, void* dst, size_t pixels, void* stream);    // rl/csrc/rlenv.cu:380-386
int rl_unpack6(const void* src, void* dst, size_t pixels, void* stream);  // rl/csrc/rlenv.cu:387-393
int rl_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);                   // rl/csrc/rlenv.cu:394-398
int rl_gather_rows(void* dst, const void* src, const int64_t* rows, int nrows, size_t row_bytes, void* stream);  // rl/csrc/rlenv.cu:400-409
int rl_gather_envs(void* dst, const void* src, const int64_t* envs, int n, int T, int N, size_t row_bytes,
                   void* stream);                                         // rl/csrc/rlenv.cu:411-421
// The reference's random legal moves (rl/actions.py:18-20 random_legal: each move part uniform among the choices its
// mask allows) on the device: masks u8[n,19] (the last decision's masks output), words u32[n] random bits (one draw
// per env; the parts' draws are mixed from it), actions i16[n] packed move ids. The distribution is the reference
// sampler's; the random stream is not torch's. Device pointers, asynchronous on `stream`.
int rl_legal_moves(const void* masks, const void* words, void* actions, int n, void* stream);

// ---------------------------------------------------------------- extensions (no reference counterpart)

// Reward parameters of one rl10 game id: 20 float64 in the order of ghostrun-lab_b200/synth.py SPEC_FIELDS
// (the reference hard-codes its 12 games' constants in rl/csrc/reward10_consts.h; synthetic games are seeded).
// Process-wide; call before rlenv_create.
int rl10_register_game(int game_id, const double* spec, int n);

// Canonical machine state of global env `ge` (CPU registers, RAM, PPU registers, nametables, palette, OAM, board
// registers and page tables, DMC, the shown frame-log bank, cartridge RAM, CHR-RAM): RLENV_DUMP_BYTES bytes into
// host memory, synchronous. The CPU oracle exports the same layout (oracle_dump_env), which the parity tests compare.
#define RLENV_DUMP_BYTES 23040
size_t rlenv_dump_bytes(void);
int rlenv_dump_env(void* h, int ge, uint8_t* host_out, void* stream);
// target, ep_frame, episode, fault, sticky counter of env ge into host memory (synchronous).
int rlenv_env_scalars(void* h, int ge, uint64_t* host_out, void* stream);
// How the pictures since the last reset were drawn (synchronous on `stream`; reset != 0 clears the counts
// afterwards): out[0] = frames the sequential renderer drew (more than 4 palette or CHR-page versions, a write inside
// a line's drawn part on the boards without split-line drawing, sprites switched on in the hblank of a line drawn with
// rendering off, every MMC2 frame), out[1] = lines with a write inside their drawn part that the two-phase renderer
// drew exactly itself (MMC3).
int rlenv_render_stats(void* h, uint64_t* host_out, int reset, void* stream);
// No counterpart in the reference. rlenv_dump_env without any device allocation, for callers that cannot allocate
// device memory: a watchdog or debugger inspecting a rollout that has spent the GPU's memory (where the staging
// allocation of rlenv_dump_env would fail), or a host whose policy fixes device memory at start-up. Dumps
// envs[0..n) (host array, 1 <= n <= RLENV_DUMP_NOALLOC_MAX_ENVS; more is rejected with a message) into host_out,
// n x RLENV_DUMP_BYTES in the rlenv_dump_env layout, synchronous on `stream`. It stages through one file-scope
// device array of 8 x RLENV_DUMP_BYTES = 184,320 bytes, which every GPU that loads the library holds until exit.
// rlenv_create does the per-device set-up while device memory is still free (the array's address by
// cudaGetSymbolAddress, and the dump kernel's code loaded), so the call itself only launches that kernel and
// copies. All calls and handles on a device share the array; calls whose work overlaps on the GPU (two threads,
// two streams) race.
#define RLENV_DUMP_NOALLOC_MAX_ENVS 8
int rlenv_dump_envs_noalloc(void* h, const int* envs, int n, uint8_t* host_out, void* stream);

// ---------------------------------------------------------------- policy input stem (rl/fused.py:163-169)

// Fused colour lookup + 2x2 stride-2 stem convolution of the policy (the reference's Triton fused_stem forward,
// rl/fused.py:36-96 and 163-169; no counterpart in the reference C-ABI): obs [B,4,224,240] colour numbers
// (packed = 0) or [B,4,224,180] 6-bit packed pictures (packed = 1, the rl_pack6 layout); emph [B,4,224]; pal4
// [512][4] bf16 = R, G, B, 0 of palette index colour | emphasis << 6; weight [16][48] bf16 (conv weight [16,12,2,2]
// flattened, k = (frame * 3 + RGB) * 4 + dy * 2 + dx); bias [16] bf16; out [B,112,120,16] bf16 channels-last.
// bf16 products, fp32 sums on the tensor cores (tcgen05). err: device int set to 1 if a tile's MMA did not complete.
// Device pointers, asynchronous on `stream`; returns non-zero on a launch error (message: rl_stem_error).
int rl_stem_fwd(const void* obs, const void* emph, const void* pal4, const void* weight, const void* bias, void* out,
                long long batch, int packed, int* err, void* stream);
const char* rl_stem_error(void);
// rl/fused.py:89-107, 130-160 (the reference's _stem_bwd_kernel / stem_bwd custom op): grad [B,112,120,16] bf16
// (the stem output's gradient, channels-last), obs / emph / pal4 / packed as for rl_stem_fwd -> dw [16][48] fp32
// (dW = sum over output pixels of grad x input^T, flattened as the forward's weight) and db [16] fp32 (sum of grad).
// work: device scratch of at least rl_stem_bwd_work_bytes() bytes (per-CTA partial sums, added in a fixed order:
// the result is deterministic). err as for rl_stem_fwd. Asynchronous on `stream`; non-zero on a bad argument.
size_t rl_stem_bwd_work_bytes(void);
int rl_stem_bwd(const void* grad, const void* obs, const void* emph, const void* pal4, void* dw, void* db,
                long long batch, int packed, void* work, size_t work_bytes, int* err, void* stream);

// No reference counterpart (the reference sums its rollout statistics in Python from the rollout buffers,
// rl/train.py:450): acc = device float64[4] to which every later decision adds the finished episodes' count, their
// deaths, their returns and the level events (added by the finishing kernel, no extra launch; the order of the fp64
// additions varies, so the return sum may differ in its last bits between runs). NULL stops it. Takes effect at the
// next call.
void rlenv_bind_episode_counters(void* h, double* acc);

// Per-kernel device time (CUDA events on the launching stream) and launch counts, for benchmarks.
void rlenv_set_timing(void* h, int on);
// Which kernel kinds rlenv_set_timing times (bit k = out13[k]'s kind: 0 frames, 1 render, 2 finish, 3 restart frames,
// 4 restart render, 5 pack6; default all): each timed launch adds two CUDA events to its stream.
void rlenv_set_timing_kinds(void* h, unsigned mask);
int rlenv_timing(void* h, double* out13, int reset);

#ifdef __cplusplus
}
#endif
