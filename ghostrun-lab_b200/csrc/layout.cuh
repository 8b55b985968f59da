// Device-side data layout of the batched NES environment (B200, sm_100a).
//
// Every per-env machine array lives in HBM in one of two layouts, chosen by who touches it most:
//   * env-minor 32-bit words, `a[word * Np + env]`: CPU registers, PPU scalars, board registers, CPU RAM and
//     cartridge RAM. The interpreter runs one env per thread; envs of a warp execute the same 6502 code, so the
//     same RAM address across 32 lanes is one 128-byte transaction.
//   * env-major bytes, `a[env * bytes + k]`: OAM, nametable RAM, palette, CHR-RAM, the frame log and the
//     per-frame presentation snapshots. The renderer runs one warp per (env, frame) and reads one env's rows
//     contiguously.
// Np = number of env slots rounded up to a multiple of 32 (a warp never straddles the array's end).
#pragma once
#include <cstdint>

namespace gr {

using u8 = std::uint8_t;
using u16 = std::uint16_t;
using u32 = std::uint32_t;
using u64 = std::uint64_t;
using i32 = std::int32_t;

// ---------------------------------------------------------------- NES timing (rl/csrc/nes_machine.cuh:28-31)
constexpr u32 kDots = 341, kLines = 262, kFrameDots = kDots * kLines;
constexpr u32 kVblankDot = 241 * kDots + 1;
constexpr u32 kPreRenderDot = 261 * kDots + 1;
constexpr u32 kVblankFlagDot = kVblankDot - 12;
constexpr u32 kStatusClearDot = kPreRenderDot - 12;
constexpr u32 kMmc3VisibleClock = 266, kMmc3PreClock = 256;
constexpr int kFceummOffset = 11;
constexpr u32 kBudget = 200000;   // instructions per frame

// ---------------------------------------------------------------- frame log (patch:969-999)
constexpr u32 kLogHdr = 16, kLogEv = 256, kLogBankWords = kLogHdr + 2 * kLogEv;   // 528 words
constexpr u32 kLogBanks = 4;   // ring: the 4 frames of a decision keep their logs until they are drawn
constexpr u32 kLogOverflow = 0x80000000u, kLogKook = 0x100u;
// log_ctl byte: bits 0-1 shown bank, bit 2 next frame is a kook frame, bit 3 the current frame is shortened
constexpr u32 kLcBank = 3u, kLcNextKook = 4u, kLcShort = 8u;
enum : u32 { kEvCtrl = 1, kEvMask, kEvScroll, kEvAddr, kEvDataWrite, kEvDataRead, kEvPalette, kEvChr, kEvMirror,
             kEvMmc2 };
constexpr u32 kS0Evaluate = 0x80000000u, kS0Known = 0x40000000u, kS0Hit = 0x20000000u, kS0DotMask = 0x1FFFFu;
constexpr u64 kDmcIdle = ~0ull;

// ---------------------------------------------------------------- boards
enum Board : u32 { kNrom = 0, kUxrom = 1, kMmc1 = 2, kMmc3 = 3, kCnrom = 4, kMmc2 = 5 };
// Boards with per-env page tables (CHR 1 KB pages, PRG 8 KB pages) and a nametable page map.
__host__ __device__ constexpr bool board_paged(u32 b) { return b == kMmc1 || b == kMmc3 || b == kCnrom || b == kMmc2; }
constexpr u8 kPageVertical = 0x0A, kPageHorizontal = 0x0C, kPageSingleLow = 0x00, kPageSingleHigh = 0x0F;

// ---------------------------------------------------------------- observation geometry
constexpr int kFramesPerDecision = 4, kObsW = 240, kObsH = 224, kObsX0 = 8, kObsY0 = 8;
constexpr int kObsPixels = kObsW * kObsH;
constexpr int kMaskBytes = 19, kDropInputs = 8, kTimeline = 45, kTimelineBytes = kDropInputs * kTimeline;
constexpr int kInfo = 8, kParts = 7, kRing = 64;

// ---------------------------------------------------------------- per-env register words (env-minor)
enum RegWord : int {
    R_PC_SP_P = 0,   // pc | sp << 16 | p << 24
    R_AXY_PAD,       // a | x << 8 | y << 16 | pad << 24
    R_CYC_LO, R_CYC_HI,
    R_FDOT,          // PPU frame dot
    R_FRAME_LO, R_FRAME_HI,
    R_PPU0,          // ctrl | mask << 8 | status << 16 | oam_addr << 24
    R_PPU1,          // nmi_pending | fine x << 8 | w << 16 | open_bus << 24
    R_PPU2,          // read_buffer | log_ctl << 8 | prg_bank << 16 | mirroring << 24
    R_VT,            // v | t << 16
    R_S0,            // sprite-0 schedule (patch:1944-1955 encoding)
    R_LOGN,          // log count | scroll_x << 16 | scroll_y << 24
    R_IO,            // controller shift | count << 8 | strobe << 16 | irq line << 24
    R_MREG,          // 4 words: board registers[16]
    R_PRGPG = R_MREG + 4,    // 4 words: 8 KB PRG page offsets
    R_CHRPG = R_PRGPG + 4,   // 8 words: 1 KB CHR page offsets
    R_DMC_END = R_CHRPG + 8, // 2 words: DMC byte_end
    R_DMC_A = R_DMC_END + 2, // bytes_left | control << 16 | length << 24
    R_DMC_B,                 // rate | buffer_full << 8
    R_DMC_EV,                // 2 words: DMC event cycle
    R_FSLOT = R_DMC_EV + 2,  // presentation slot holding the last frozen frame (0..3)
    R_CHRD,                  // CHR-RAM carts: 1 = CHR-RAM written since the env's shared CHR snapshot was taken
    kRegWords
};

constexpr u32 kRamWords = 512, kPrgRamWords = 2048;
constexpr u32 kOamBytes = 256, kNtBytes = 2048, kPalBytes = 32, kChrRamBytes = 8192;

// Canonical per-env dump (same bytes as the CPU oracle's): see include/rlenv_api.h.
constexpr u32 kDumpBytes = 23040;

// One console's whole state as a flat record (boot / idle snapshots, state save): register words, RAM, cartridge
// RAM, OAM, nametables, palette, CHR-RAM, the shown frame-log bank and the frozen nametable/OAM it is drawn from.
constexpr u32 kRecRegs = 0;
constexpr u32 kRecRam = kRecRegs + 4 * 64;
constexpr u32 kRecPrgRam = kRecRam + 2048;
constexpr u32 kRecOam = kRecPrgRam + 8192;
constexpr u32 kRecNt = kRecOam + 256;
constexpr u32 kRecPal = kRecNt + 2048;
constexpr u32 kRecChrRam = kRecPal + 32;
constexpr u32 kRecLog = kRecChrRam + 8192;
constexpr u32 kRecSnapNt = kRecLog + kLogBanks * kLogBankWords * 4;
constexpr u32 kRecSnapOam = kRecSnapNt + 2048;
constexpr u32 kRecBytes = kRecSnapOam + 256;
static_assert(kRegWords <= 64, "register words must fit the record header");
static_assert(kRecBytes % 16 == 0, "records are copied in 16-byte vectors");

// ---------------------------------------------------------------- reward spec (ghostrun-lab_b200/synth.py order)
struct Spec {
    double progress_unit, score_unit, stall_frames, idle_per_frame, death_from_lives, start_ok, select_ok;
    double w_progress, w_level, w_death, w_damage, w_score, score_cap, score_level_budget, w_win, w_stall,
        w_rollback, rollback_drop, reader, frame_limit;
};
constexpr int kSpecFields = 20;

// ---------------------------------------------------------------- device views

struct CartView {
    const u8* prg;       // padded to a power of two
    u32 prg_mask;
    const u8* chr;       // CHR ROM, nullptr = CHR-RAM
    u32 chr_size;
    const u32* chrx;     // CHR ROM as 4-bit-per-pixel rows: chrx[row * tiles + tile] (see render.cuh)
    u32 chr_tiles;
    u32 board, arrangement;
    u32 bank_mask, fixed_base, prg_page_mask, chr_page_mask;
    // PRG window staged in each emulation block's shared memory: bytes [prg_stage_base, + prg_stage_bytes) of prg
    // (the whole PRG on NROM, the last 16 KB - the fixed bank the reset / NMI code runs from - on the paged boards)
    u32 prg_stage_base, prg_stage_bytes;
};
constexpr u32 kPrgStageMax = 32768;

struct StateView {
    u32 Np;
    u32* regs;       // [kRegWords][Np]
    u32* ram;        // [512][Np]
    u32* prg_ram;    // [2048][Np]
    u8* oam;         // [Np][256]
    u8* nt;          // [Np][2048]
    u8* pal;         // [Np][32]
    u8* chr_ram;     // [Np][8192] (CHR-RAM carts), else nullptr
    u32* log;        // [Np][kLogBanks][528]
    u8* snap_nt;     // [Np][4][2048] nametable RAM frozen at each frame's vblank
    u8* snap_oam;    // [Np][4][256]
    u8* snap_chr;    // [Np][4][8192] (CHR-RAM carts)
    // CHR-RAM carts: one shared snapshot per env, taken when a launch starts with CHR-RAM written since the last one;
    // a frame frozen with no CHR-RAM write since then points at it (chr_ref = 1) instead of copying 8 KB
    u8* chr_shared;  // [Np][8192], nullptr: every slot keeps its own copy
    u8* chr_ref;     // [Np][4]
    u8* slot_bank;   // [Np][4] frame-log bank shown by presentation slot f
};

// Reward / RL per-env state (one 128-byte record per env).
struct Tracker {   // RewardTracker + Signals of the previous update
    double best_progress, score_used, prev_progress, prev_health;
    long long idle_frames, prev_score;
    i32 best_level, deaths, prev_level, prev_lives;
    u8 has_prev, has_best_level, has_best_progress, done, end_reason, overflow;
    u8 prev_in_play, prev_progress_valid, prev_dying, prev_has_lives, prev_has_health, prev_has_score,
        prev_game_over, prev_won;
};

struct Dropout {
    u64 seed, counter;
    i32 gap_left, drop_left, drop_input;
    u32 head;
    int8_t ring[kRing];
};

}  // namespace gr
