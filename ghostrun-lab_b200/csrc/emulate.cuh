// Thread-per-env NES emulation for sm_100a: the 6502 interpreter, the CPU bus, lazy PPU timing, the frame log and
// the sprite-0 hit, specialised per board at compile time.
//
// Behaviour follows the reference environment's emulator (NeSLE batch code as patched by
// third_party/nesle-extensions.patch, driven by rl/csrc/nes_machine.cuh:67-103):
//   * frame loop, lazy settle, JMP-to-self fast-forward, 200k-instruction budget  (nes_machine.cuh:67-103)
//   * instruction step with NMI / level IRQ, frame-log cycle stamps, DMA stall, DMC steals  (patch:834-893)
//   * PPU events: early vblank flag, NMI, status clear, pre-render capture, sprite-0, short frames, MMC3 clocks
//     (patch:1857-2240)
//   * frame log recording (patch:1047-1185) and PPU / board bus hooks (patch:570-780)
// The 6502 core, $2002/$2004/$2007 reads, OAM DMA length, the controller port and the UxROM window belong to the
// NeSLE base tree, which is not vendored; they follow public 6502/NES documentation and the definitions the CPU
// oracle states (oracle/nes.hpp), and the two are held bit-exact by tests.
//
// Design for the GPU: one env per thread; the opcode is decoded through a 256-entry table in shared memory into
// (addressing mode, operation, cycles), so lanes that run different instructions still share the addressing and
// memory stages; CPU RAM is env-minor so a warp's lanes touching the same address coalesce.
#pragma once
#include "layout.cuh"

namespace gr {

enum : u32 { FC = 1, FZ = 2, FI = 4, FD = 8, FB = 0x10, FU = 0x20, FV = 0x40, FN = 0x80 };

// ------------------------------------------------------------------------------------------------ decode table
// entry: mode (4 bits) | op << 4 (6 bits) | cycles << 10 (4 bits) | page-cross penalty << 14, and the addressing
// mode's effective-address recipe for a branch-free computation: length - 1 << 15 (2 bits), index X (bit 17) or Y
// (bit 18), zero-page wrap (bit 19), 16-bit operand (bit 20), indirect (bit 21: (zp,X), (zp),Y, JMP (ind))
enum Mode : u32 { M_IMP = 0, M_ACC, M_IMM, M_ZP, M_ZPX, M_ZPY, M_ABS, M_ABSX, M_ABSY, M_IND, M_INDX, M_INDY, M_REL };
enum Op : u32 {
    O_ILL = 0, O_LDA, O_LDX, O_LDY, O_STA, O_STX, O_STY, O_ADC, O_SBC, O_AND, O_ORA, O_EOR, O_CMP, O_CPX, O_CPY,
    O_BIT, O_ASL, O_LSR, O_ROL, O_ROR, O_INC, O_DEC, O_INX, O_INY, O_DEX, O_DEY, O_TAX, O_TAY, O_TXA, O_TYA, O_TSX,
    O_TXS, O_CLC, O_SEC, O_CLI, O_SEI, O_CLV, O_CLD, O_SED, O_NOP, O_PHA, O_PHP, O_PLA, O_PLP, O_JMP, O_JSR, O_RTS,
    O_RTI, O_BRK, O_BPL, O_BMI, O_BVC, O_BVS, O_BCC, O_BCS, O_BNE, O_BEQ
};

enum : u32 { kDLen = 15, kDX = 1u << 17, kDY = 1u << 18, kDZp = 1u << 19, kDAbs = 1u << 20, kDInd = 1u << 21 };
constexpr u32 mode_bits(u32 mode) {
    switch (mode) {
        case M_IMP: case M_ACC: return 0u << kDLen;
        case M_IMM: case M_REL: return 1u << kDLen;
        case M_ZP: return (1u << kDLen) | kDZp;
        case M_ZPX: return (1u << kDLen) | kDZp | kDX;
        case M_ZPY: return (1u << kDLen) | kDZp | kDY;
        case M_ABS: return (2u << kDLen) | kDAbs;
        case M_ABSX: return (2u << kDLen) | kDAbs | kDX;
        case M_ABSY: return (2u << kDLen) | kDAbs | kDY;
        case M_IND: return (2u << kDLen) | kDAbs | kDInd;
        case M_INDX: return (1u << kDLen) | kDInd | kDX;
        default: return (1u << kDLen) | kDInd | kDY;   // M_INDY
    }
}
constexpr u32 dec(u32 mode, u32 op, u32 cyc, u32 px = 0) {
    return mode | (op << 4) | (cyc << 10) | (px << 14) | mode_bits(mode);
}

struct DecodeTable {
    u32 t[256];
    constexpr DecodeTable() : t{} {
        for (int i = 0; i < 256; ++i) t[i] = 0;
        // group 1: ORA AND EOR ADC STA LDA CMP SBC by (op >> 2) & 7 = (zp,X) zp imm abs (zp),Y zp,X abs,Y abs,X
        const u32 g1[8] = {O_ORA, O_AND, O_EOR, O_ADC, O_STA, O_LDA, O_CMP, O_SBC};
        const u32 m1[8] = {M_INDX, M_ZP, M_IMM, M_ABS, M_INDY, M_ZPX, M_ABSY, M_ABSX};
        const u32 c1[8] = {6, 3, 2, 4, 5, 4, 4, 4};
        for (u32 a = 0; a < 8; ++a)
            for (u32 b = 0; b < 8; ++b) {
                const u32 opc = (a << 5) | (b << 2) | 1;
                if (g1[a] == O_STA) {
                    if (b == 2) continue;
                    const u32 sc[8] = {6, 3, 0, 4, 6, 4, 5, 5};
                    t[opc] = dec(m1[b], O_STA, sc[b]);
                } else {
                    t[opc] = dec(m1[b], g1[a], c1[b], (b == 4 || b == 6 || b == 7) ? 1 : 0);
                }
            }
        // read-modify-write: ASL ROL LSR ROR (+DEC INC) on zp / abs / zp,X / abs,X and the accumulator forms
        const u32 g2[8] = {O_ASL, O_ROL, O_LSR, O_ROR, 0, 0, O_DEC, O_INC};
        for (u32 a = 0; a < 8; ++a) {
            if (!g2[a]) continue;
            t[(a << 5) | 0x06] = dec(M_ZP, g2[a], 5);
            t[(a << 5) | 0x0E] = dec(M_ABS, g2[a], 6);
            t[(a << 5) | 0x16] = dec(M_ZPX, g2[a], 6);
            t[(a << 5) | 0x1E] = dec(M_ABSX, g2[a], 7);
            if (a < 4) t[(a << 5) | 0x0A] = dec(M_ACC, g2[a], 2);
        }
        t[0xA2] = dec(M_IMM, O_LDX, 2); t[0xA6] = dec(M_ZP, O_LDX, 3); t[0xB6] = dec(M_ZPY, O_LDX, 4);
        t[0xAE] = dec(M_ABS, O_LDX, 4); t[0xBE] = dec(M_ABSY, O_LDX, 4, 1);
        t[0xA0] = dec(M_IMM, O_LDY, 2); t[0xA4] = dec(M_ZP, O_LDY, 3); t[0xB4] = dec(M_ZPX, O_LDY, 4);
        t[0xAC] = dec(M_ABS, O_LDY, 4); t[0xBC] = dec(M_ABSX, O_LDY, 4, 1);
        t[0x86] = dec(M_ZP, O_STX, 3); t[0x96] = dec(M_ZPY, O_STX, 4); t[0x8E] = dec(M_ABS, O_STX, 4);
        t[0x84] = dec(M_ZP, O_STY, 3); t[0x94] = dec(M_ZPX, O_STY, 4); t[0x8C] = dec(M_ABS, O_STY, 4);
        t[0xE0] = dec(M_IMM, O_CPX, 2); t[0xE4] = dec(M_ZP, O_CPX, 3); t[0xEC] = dec(M_ABS, O_CPX, 4);
        t[0xC0] = dec(M_IMM, O_CPY, 2); t[0xC4] = dec(M_ZP, O_CPY, 3); t[0xCC] = dec(M_ABS, O_CPY, 4);
        t[0x24] = dec(M_ZP, O_BIT, 3); t[0x2C] = dec(M_ABS, O_BIT, 4);
        t[0xE8] = dec(M_IMP, O_INX, 2); t[0xC8] = dec(M_IMP, O_INY, 2); t[0xCA] = dec(M_IMP, O_DEX, 2);
        t[0x88] = dec(M_IMP, O_DEY, 2); t[0xAA] = dec(M_IMP, O_TAX, 2); t[0xA8] = dec(M_IMP, O_TAY, 2);
        t[0x8A] = dec(M_IMP, O_TXA, 2); t[0x98] = dec(M_IMP, O_TYA, 2); t[0xBA] = dec(M_IMP, O_TSX, 2);
        t[0x9A] = dec(M_IMP, O_TXS, 2); t[0x18] = dec(M_IMP, O_CLC, 2); t[0x38] = dec(M_IMP, O_SEC, 2);
        t[0x58] = dec(M_IMP, O_CLI, 2); t[0x78] = dec(M_IMP, O_SEI, 2); t[0xB8] = dec(M_IMP, O_CLV, 2);
        t[0xD8] = dec(M_IMP, O_CLD, 2); t[0xF8] = dec(M_IMP, O_SED, 2); t[0xEA] = dec(M_IMP, O_NOP, 2);
        t[0x48] = dec(M_IMP, O_PHA, 3); t[0x08] = dec(M_IMP, O_PHP, 3); t[0x68] = dec(M_IMP, O_PLA, 4);
        t[0x28] = dec(M_IMP, O_PLP, 4); t[0x4C] = dec(M_ABS, O_JMP, 3); t[0x6C] = dec(M_IND, O_JMP, 5);
        t[0x20] = dec(M_ABS, O_JSR, 6); t[0x60] = dec(M_IMP, O_RTS, 6); t[0x40] = dec(M_IMP, O_RTI, 6);
        t[0x00] = dec(M_IMP, O_BRK, 7);
        t[0x10] = dec(M_REL, O_BPL, 2); t[0x30] = dec(M_REL, O_BMI, 2); t[0x50] = dec(M_REL, O_BVC, 2);
        t[0x70] = dec(M_REL, O_BVS, 2); t[0x90] = dec(M_REL, O_BCC, 2); t[0xB0] = dec(M_REL, O_BCS, 2);
        t[0xD0] = dec(M_REL, O_BNE, 2); t[0xF0] = dec(M_REL, O_BEQ, 2);
    }
};
static __constant__ DecodeTable kDecode = DecodeTable();

// ------------------------------------------------------------------------------------------------ small helpers

__device__ __forceinline__ int fceumm_time(u32 dot, int kook) {
    const int d = static_cast<int>(dot);
    return dot >= kPreRenderDot ? d - static_cast<int>(kFrameDots) + kFceummOffset + kook : d + kFceummOffset;
}
__device__ __forceinline__ u32 nesle_dot(int f) { return static_cast<u32>(f - kFceummOffset); }

__device__ __forceinline__ u32 dmc_period(u32 rate) {
    // NTSC CPU cycles per DMC output bit, $4010 bits 0-3
    const u32 lo = 0u;
    (void)lo;
    switch (rate & 15) {
        case 0: return 428; case 1: return 380; case 2: return 340; case 3: return 320;
        case 4: return 286; case 5: return 254; case 6: return 226; case 7: return 214;
        case 8: return 190; case 9: return 160; case 10: return 142; case 11: return 128;
        case 12: return 106; case 13: return 84; case 14: return 72; default: return 54;
    }
}

// CIRAM offset of a $2000-$3EFF address for header mirroring (non-paged boards) or a page map (paged).
__device__ __forceinline__ u32 nt_off_header(u32 arrangement, u32 addr) {
    const u32 index = (addr - 0x2000u) & 0x0FFFu;
    return arrangement == 1 ? ((((index >> 11) & 1u) << 10) | (index & 0x3FFu)) : (index & 0x7FFu);
}
__device__ __forceinline__ u32 nt_off_map(u32 map, u32 addr) {
    const u32 index = (addr - 0x2000u) & 0x0FFFu;
    return (((map >> (index >> 10)) & 1u) << 10) | (index & 0x3FFu);
}

// Coarse-x / fine-y increments of the PPU address (FCEUmm's tile loop and Fixit1).
__device__ __forceinline__ u32 v_inc_x(u32 v) { return ((v & 0x1Fu) == 0x1Fu) ? (v ^ 0x41Fu) : (v + 1u); }
__device__ __forceinline__ u32 v_inc_x_n(u32 v, u32 n) {   // n increments (n <= 64)
    const u32 c = (v & 0x1Fu) + n;
    return (v & ~0x41Fu) | (((v & 0x400u) ^ (((c >> 5) & 1u) << 10))) | (c & 0x1Fu);
}
__device__ __forceinline__ u32 v_inc_y(u32 v) {
    if ((v & 0x7000u) == 0x7000u) {
        v ^= 0x7000u;
        if ((v & 0x3E0u) == 0x3A0u) v ^= 0xBA0u;
        else if ((v & 0x3E0u) == 0x3E0u) v ^= 0x3E0u;
        else v += 0x20u;
    } else {
        v += 0x1000u;
    }
    return v & 0x7FFFu;
}
// v after k line ends without events (k <= 240): the vertical increment k times (coarse Y 29 -> 0 toggles the
// vertical nametable, 31 -> 0 does not), the horizontal bits from t (th) once k >= 1; rendering off: v stays.
__device__ __forceinline__ u32 v_after_lines(u32 v, u32 k, u32 th, bool ren) {
    if (k == 0 || !ren) return v;
    u32 y = ((v >> 5) & 31u) * 8u + ((v >> 12) & 7u);
    u32 nty = v & 0x800u;
    y += k;
    if (y - k < 240u) {
        if (y >= 240u) { y -= 240u; nty ^= 0x800u; }
    } else if (y >= 256u) {
        y -= 256u;
        if (y >= 240u) { y -= 240u; nty ^= 0x800u; }
    }
    return th | nty | ((y & 7u) << 12) | ((y >> 3) << 5);
}

// ------------------------------------------------------------------------------------------------ emulator

struct Hit0 { u32 dot; bool hit; };

// Consoles per warp in the emulation kernels: lanes 0..kEnvsPerWarp-1 each run one console, the others idle. Fewer
// consoles per warp mean fewer distinct program counters per min-PC round and more warps, but each warp runs the
// whole interpreter body per round: measured, 2 warps x 16 beat 1 x 32 by 3-6% on NROM / UxROM / MMC1 run alone but
// lost 5% on MMC3 and on the mixed config-3 run; 8 x 4 and 4 x 8 lost everywhere. A board unit may set both before
// including this header (board_nrom.cu does).
#ifndef GR_ENVS_PER_WARP
#define GR_ENVS_PER_WARP 32
#endif
constexpr u32 kEnvsPerWarp = GR_ENVS_PER_WARP;
// Emulation warps per block: each stages its own consoles, the block shares one decode table and one PRG window
#ifndef GR_FRAMES_WARPS
#define GR_FRAMES_WARPS 1
#endif
constexpr u32 kFramesWarps = GR_FRAMES_WARPS;
static_assert(kEnvsPerWarp == 4 || kEnvsPerWarp == 8 || kEnvsPerWarp == 16 || kEnvsPerWarp == 32, "envs per warp");

// Shared-memory staging of one warp's consoles: register words, CPU RAM and OAM, each lane a column (word w of
// lane l at [w][l]), so every lane touches its own bank whatever addresses the lanes use.
struct EmuShared {
    u32 regs[kRegWords][kEnvsPerWarp];
    u32 ram[kRamWords][kEnvsPerWarp];
    u32 oam[64][kEnvsPerWarp];
};

template <u32 BOARD>
struct Emu {
    const StateView& S;
    const CartView& C;
    const u32 e;          // global env slot
    const u32 lane;       // column in the shared staging
    EmuShared& sh;
    const u32* __restrict__ dtab;   // decode table (shared memory)
    const u8* __restrict__ prg_s;   // the cart's staged PRG window (shared memory)
    // hot state (registers for the whole frame loop)
    u32 pc, a, x, y, sp, p, pad;
    u64 cycles;
    u32 frame_dot;
    u64 frame;
    u32 ctrl, mask, status, oam_addr, nmi;
    u32 log_n, log_ctl;
    u32 now;
    u32 pend;     // PPU dots run since frame_dot (not yet settled) during step_until
    u64 dmc_at;   // the DMC's next event cycle (register words R_DMC_EV), kept here for the per-instruction check
    u32 resched;  // MMC3: a store changed what the scanline counter does; the next event is recomputed
    u32 dma;
    u32 slot;     // presentation slot of the frame being emulated
    u32 prg_bank; // UxROM
    u32 froze;    // the vblank froze slot `slot` during this step_until (its snapshot copy is still to be made)

    __device__ Emu(const StateView& s, const CartView& c, u32 env, u32 ln, EmuShared& shm, const u32* dt, const u8* ps)
        : S(s), C(c), e(env), lane(ln), sh(shm), dtab(dt), prg_s(ps) {}

    // -------- staging: global env-minor / env-major arrays <-> this lane's shared column
    __device__ __forceinline__ void stage_in() const {
        const u64 Np = S.Np;
        for (int w = 0; w < kRegWords; ++w) sh.regs[w][lane] = S.regs[static_cast<u64>(w) * Np + e];
        for (u32 i = 0; i < kRamWords; ++i) sh.ram[i][lane] = S.ram[static_cast<u64>(i) * Np + e];
        const uint4* o = reinterpret_cast<const uint4*>(S.oam + static_cast<u64>(e) * kOamBytes);
        for (u32 i = 0; i < 16; ++i) {
            const uint4 q = o[i];
            sh.oam[4 * i][lane] = q.x; sh.oam[4 * i + 1][lane] = q.y; sh.oam[4 * i + 2][lane] = q.z; sh.oam[4 * i + 3][lane] = q.w;
        }
    }
    __device__ __forceinline__ void stage_out() const {
        const u64 Np = S.Np;
        for (int w = 0; w < kRegWords; ++w) S.regs[static_cast<u64>(w) * Np + e] = sh.regs[w][lane];
        for (u32 i = 0; i < kRamWords; ++i) S.ram[static_cast<u64>(i) * Np + e] = sh.ram[i][lane];
        uint4* o = reinterpret_cast<uint4*>(S.oam + static_cast<u64>(e) * kOamBytes);
        for (u32 i = 0; i < 16; ++i)
            o[i] = make_uint4(sh.oam[4 * i][lane], sh.oam[4 * i + 1][lane], sh.oam[4 * i + 2][lane], sh.oam[4 * i + 3][lane]);
    }

    // -------- register-word access (shared staging)
    __device__ __forceinline__ u32 rw(int w) const { return sh.regs[w][lane]; }
    __device__ __forceinline__ void ww(int w, u32 v) const { sh.regs[w][lane] = v; }
    __device__ __forceinline__ u32 field(int w, int shift, u32 maskv) const { return (rw(w) >> shift) & maskv; }
    __device__ __forceinline__ void set_field(int w, int shift, u32 maskv, u32 v) const {
        const u32 old = rw(w);
        ww(w, (old & ~(maskv << shift)) | ((v & maskv) << shift));
    }

    __device__ __forceinline__ void load() {
        const u32 w0 = rw(R_PC_SP_P), w1 = rw(R_AXY_PAD);
        pc = w0 & 0xFFFF; sp = (w0 >> 16) & 0xFF; p = w0 >> 24;
        a = w1 & 0xFF; x = (w1 >> 8) & 0xFF; y = (w1 >> 16) & 0xFF; pad = w1 >> 24;
        cycles = rw(R_CYC_LO) | (static_cast<u64>(rw(R_CYC_HI)) << 32);
        frame_dot = rw(R_FDOT);
        frame = rw(R_FRAME_LO) | (static_cast<u64>(rw(R_FRAME_HI)) << 32);
        const u32 p0 = rw(R_PPU0);
        ctrl = p0 & 0xFF; mask = (p0 >> 8) & 0xFF; status = (p0 >> 16) & 0xFF; oam_addr = p0 >> 24;
        nmi = rw(R_PPU1) & 0xFF;
        const u32 p2 = rw(R_PPU2);
        log_ctl = (p2 >> 8) & 0xFF;
        prg_bank = (p2 >> 16) & 0xFF;
        log_n = rw(R_LOGN) & 0xFFFF;
        dmc_at = rw(R_DMC_EV) | (static_cast<u64>(rw(R_DMC_EV + 1)) << 32);
        dma = 0;
        now = 0;
        pend = 0;
        resched = 0;
    }
    __device__ __forceinline__ void store() {
        ww(R_PC_SP_P, pc | (sp << 16) | (p << 24));
        ww(R_AXY_PAD, a | (x << 8) | (y << 16) | (pad << 24));
        ww(R_CYC_LO, static_cast<u32>(cycles)); ww(R_CYC_HI, static_cast<u32>(cycles >> 32));
        ww(R_FDOT, frame_dot);
        ww(R_FRAME_LO, static_cast<u32>(frame)); ww(R_FRAME_HI, static_cast<u32>(frame >> 32));
        ww(R_PPU0, ctrl | (mask << 8) | (status << 16) | (oam_addr << 24));
        set_field(R_PPU1, 0, 0xFF, nmi);
        const u32 p2 = rw(R_PPU2);
        ww(R_PPU2, (p2 & 0xFF0000FFu) | (log_ctl << 8) | (prg_bank << 16));
        set_field(R_LOGN, 0, 0xFFFF, log_n);
    }

    // -------- memories
    __device__ __forceinline__ u32 ram_rd(u32 addr) const {
        addr &= 0x7FFu;
        return reinterpret_cast<const u8*>(&sh.ram[addr >> 2][lane])[addr & 3u];
    }
    __device__ __forceinline__ void ram_wr(u32 addr, u32 v) const {
        addr &= 0x7FFu;
        reinterpret_cast<u8*>(&sh.ram[addr >> 2][lane])[addr & 3u] = static_cast<u8>(v);
    }
    __device__ __forceinline__ u8* prgram8() const { return reinterpret_cast<u8*>(S.prg_ram); }
    __device__ __forceinline__ u64 prgram_index(u32 off) const {
        return ((static_cast<u64>(off >> 2) * S.Np + e) << 2) | (off & 3u);
    }
    __device__ __forceinline__ u32 oam_rd(u32 i) const { return reinterpret_cast<const u8*>(&sh.oam[i >> 2][lane])[i & 3u]; }
    __device__ __forceinline__ void oam_wr(u32 i, u32 v) const { reinterpret_cast<u8*>(&sh.oam[i >> 2][lane])[i & 3u] = static_cast<u8>(v); }
    __device__ __forceinline__ u8* nt() const { return S.nt + static_cast<u64>(e) * kNtBytes; }
    __device__ __forceinline__ u8* pal() const { return S.pal + static_cast<u64>(e) * kPalBytes; }
    __device__ __forceinline__ u8* chr_ram() const { return S.chr_ram + static_cast<u64>(e) * kChrRamBytes; }
    __device__ __forceinline__ u32* log_bank(u32 b) const {
        return S.log + (static_cast<u64>(e) * kLogBanks + (b & 3u)) * kLogBankWords;
    }
    __device__ __forceinline__ u32* writing_bank() const { return log_bank((log_ctl & kLcBank) + 1u); }

    __device__ __forceinline__ u32 mreg(u32 i) const { return (rw(R_MREG + (i >> 2)) >> ((i & 3) * 8)) & 0xFF; }
    __device__ __forceinline__ void set_mreg(u32 i, u32 v) const { set_field(R_MREG + (i >> 2), (i & 3) * 8, 0xFF, v); }
    __device__ __forceinline__ u32 mirroring() const { return rw(R_PPU2) >> 24; }

    __device__ __forceinline__ u32 prg_byte(u32 off) const {   // PRG byte at physical offset off
        const u32 k = off - C.prg_stage_base;
        return k < C.prg_stage_bytes ? static_cast<u32>(prg_s[k]) : static_cast<u32>(__ldg(C.prg + off));
    }
    __device__ __forceinline__ u32 prg_rd(u32 addr) const {
        if constexpr (BOARD == kNrom || BOARD == kCnrom) {   // 16 / 32 KB fixed (CNROM's PRG pages are 0-3)
            return prg_s[(addr - 0x8000u) & C.prg_mask];   // the whole PRG is staged
        } else if constexpr (BOARD == kUxrom) {
            const u32 off = addr < 0xC000u ? (((prg_bank & C.bank_mask) << 14) | (addr & 0x3FFFu))
                                           : (C.fixed_base + (addr & 0x3FFFu));
            return prg_byte(off);
        } else {
            return prg_byte(rw(R_PRGPG + ((addr >> 13) & 3u)) + (addr & 0x1FFFu));
        }
    }

    __device__ __forceinline__ u32 chr_rd(u32 addr) const {
        addr &= 0x1FFFu;
        if constexpr (board_paged(BOARD)) {
            const u32 off = rw(R_CHRPG + (addr >> 10)) + (addr & 0x3FFu);
            return C.chr ? __ldg(C.chr + off) : chr_ram()[off & 0x1FFFu];
        } else {
            return C.chr ? __ldg(C.chr + (addr % C.chr_size)) : chr_ram()[addr];
        }
    }
    __device__ __forceinline__ void chr_wr(u32 addr, u32 v) const {
        if (C.chr) return;
        addr &= 0x1FFFu;
        if constexpr (board_paged(BOARD)) addr = (rw(R_CHRPG + (addr >> 10)) + (addr & 0x3FFu)) & 0x1FFFu;
        chr_ram()[addr] = static_cast<u8>(v);
        ww(R_CHRD, 1u);
    }
    __device__ __forceinline__ u32 nt_off(u32 addr) const {
        if constexpr (board_paged(BOARD)) return nt_off_map(mirroring(), addr);
        else return nt_off_header(C.arrangement, addr);
    }
    __device__ __forceinline__ static u32 pal_index(u32 addr) {
        u32 i = addr & 0x1Fu;
        if ((i & 0x13u) == 0x10u) i &= 0x0Fu;
        return i;
    }
    __device__ __forceinline__ u32 ppu_mem_rd(u32 addr) const {
        addr &= 0x3FFFu;
        if (addr < 0x2000u) return chr_rd(addr);
        if (addr < 0x3F00u) return nt()[nt_off(addr >= 0x3000u ? addr - 0x1000u : addr)];
        return pal()[pal_index(addr)];
    }
    __device__ __forceinline__ void ppu_mem_wr(u32 addr, u32 v) const {
        addr &= 0x3FFFu;
        if (addr < 0x2000u) { chr_wr(addr, v); return; }
        if (addr < 0x3F00u) { nt()[nt_off(addr >= 0x3000u ? addr - 0x1000u : addr)] = static_cast<u8>(v); return; }
        pal()[pal_index(addr)] = static_cast<u8>(v);
    }

    // -------- frame log
    __device__ __forceinline__ bool log_active() const { return now < kVblankDot || now >= kPreRenderDot; }

    __device__ __forceinline__ void log_event(u32 kind, u32 value, u32 aux) {
        if (!log_active()) return;
        u32* bank = writing_bank();
        if (kind == kEvDataWrite && (mask & 0x18u) == 0 && log_n != 0 && log_n <= kLogEv) {
            u32* last = bank + kLogHdr + 2 * (log_n - 1);
            if ((last[0] >> 24) == kEvDataWrite && (last[1] >> 8) < 0xFFu) { last[1] += 0x100u; return; }
        }
        if (log_n >= kLogEv) { bank[0] |= kLogOverflow; return; }
        u32* ev = bank + kLogHdr + 2 * log_n;
        ev[0] = (now & 0x1FFFFu) | (kind << 24);
        ev[1] = (value & 0xFFu) | ((aux & 0xFFu) << 8);
        ++log_n;
    }

    __device__ __forceinline__ void fill_header(u32* h) const {
        const u32 vt = rw(R_VT);
        const u32 fx = (rw(R_PPU1) >> 8) & 7u;
        uint4 w0, w1, w2, w3;
        w0.x = 0;
        w0.y = ctrl | (mask << 8) | (fx << 16);
        w0.z = (vt & 0xFFFFu) | ((vt >> 16) << 16);
        w0.w = 0;
        w1.x = 0; w1.y = 0; w1.z = 0;
        if constexpr (board_paged(BOARD)) {
            u32 c0 = 0, c1 = 0;
            for (u32 i = 0; i < 4; ++i) c0 |= ((rw(R_CHRPG + i) >> 10) & 0xFFu) << (i * 8);
            for (u32 i = 0; i < 4; ++i) c1 |= ((rw(R_CHRPG + 4 + i) >> 10) & 0xFFu) << (i * 8);
            w0.w = c0; w1.x = c1; w1.y = mirroring();
            if constexpr (BOARD == kMmc2) {   // latches in h[5], the four CHR registers in h[6] (patch:1034-1040)
                w1.y |= ((mreg(6) & 1u) << 8) | ((mreg(7) & 1u) << 16);
                w1.z = rw(R_MREG);
            }
        }
        const uint4* pp = reinterpret_cast<const uint4*>(pal());
        const uint4 pa = pp[0], pb = pp[1];
        w1.w = pa.x;
        w2.x = pa.y; w2.y = pa.z; w2.z = pa.w; w2.w = pb.x;
        w3.x = pb.y; w3.y = pb.z; w3.z = pb.w; w3.w = 0;
        uint4* hv = reinterpret_cast<uint4*>(h);
        hv[0] = w0; hv[1] = w1; hv[2] = w2; hv[3] = w3;
    }

    // pre-render: the writing bank starts over from the live state (patch:1080-1088)
    __device__ __forceinline__ void log_capture() {
        u32* h = writing_bank();
        fill_header(h);
        const bool kook = (log_ctl & kLcNextKook) != 0;
        if (kook) h[15] = kLogKook;
        log_ctl = ((log_ctl ^ kLcNextKook) & ~kLcShort) | (kook ? kLcShort : 0u);
        log_n = 0;
    }

    // FCEUmm's emphasis tint after the frame in `h` (patch:1087-1118)
    __device__ __forceinline__ static u32 emphasis(const u32* h, u32 previous) {
        const u32* ev = h + kLogHdr;
        const u32 count = h[0] & ~kLogOverflow;
        u32 m = (h[1] >> 8) & 0xFFu;
        if (count == 0) {   // one mask for every line: its emphasis if it is 1..6, else the previous tint
            const u32 d = m >> 5;
            return (d >= 1 && d <= 6) ? d : previous;
        }
        bool any = (m & 0xE0u) != 0;
        for (u32 i = 0; i < count && !any; ++i) any = (ev[2 * i] >> 24) == kEvMask && (ev[2 * i + 1] & 0xE0u) != 0;
        if (!any) return previous;
        const int kook = (h[15] & kLogKook) ? 1 : 0;
        u32 i = 0;
        for (; i < count && fceumm_time(ev[2 * i] & 0x1FFFFu, kook) < 0; ++i)
            if ((ev[2 * i] >> 24) == kEvMask) m = ev[2 * i + 1] & 0xFFu;
        u32 deemp = m >> 5;
        u32 lines[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int l = 0; l < 240; ++l) {
            for (; i < count && fceumm_time(ev[2 * i] & 0x1FFFFu, kook) < l * 341; ++i) {
                const u32 value = ev[2 * i + 1] & 0xFFu;
                if ((ev[2 * i] >> 24) == kEvMask && (value & 0xE0u)) deemp = value >> 5;
            }
            ++lines[deemp];
        }
        u32 most = 0, best = 0;
        for (u32 k = 1; k < 7; ++k) if (lines[k] > most) { most = lines[k]; best = k; }
        return best ? best : previous;
    }

    // Copy 16-byte vectors (both pointers 16-byte aligned).
    __device__ __forceinline__ static void copy16(u8* dst, const u8* src, u32 bytes) {   // bytes: a multiple of 128
        uint4* d = reinterpret_cast<uint4*>(dst);
        const uint4* s = reinterpret_cast<const uint4*>(src);
        for (u32 i = 0; i < bytes / 16; i += 8) {
            uint4 q[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) q[k] = s[i + k];
#pragma unroll
            for (int k = 0; k < 8; ++k) d[i + k] = q[k];
        }
    }

    // vblank: the writing bank becomes the shown one, and the nametable RAM / OAM (/ CHR-RAM) it is drawn from are
    // frozen into this frame's presentation slot (patch:1121-1130, 2487-2520)
    __device__ __forceinline__ void log_freeze() {
        const u32 shown = log_ctl & kLcBank;
        u32* h = writing_bank();
        const u32* old = log_bank(shown);
        h[0] = (h[0] & kLogOverflow) | log_n;
        h[15] = (h[15] & ~7u) | emphasis(h, old[15] & 7u);
        const u32 nb = (shown + 1u) & kLcBank;
        log_ctl = (log_ctl & ~kLcBank) | nb;
        const u64 sl = static_cast<u64>(e) * 4 + slot;
        froze = 1;    // the vblank ends the frame's step_until: snapshot_frozen copies the memories after it
        S.slot_bank[sl] = static_cast<u8>(nb);
        ww(R_FSLOT, slot);
    }

    // After step_until (all 32 lanes): the nametable RAM, OAM (and CHR-RAM) of every lane that froze a frame into
    // presentation slot `slot`, copied by the whole warp. Nothing runs between the vblank and the end of the frame's
    // step_until (the frame's target is the vblank dot), so the memories are still as frozen.
    // At a launch's start (all 32 lanes): envs whose CHR-RAM was written since their shared CHR snapshot take a new
    // one. No slot of the frames to come points at the old one yet, and earlier slots have been drawn.
    __device__ __forceinline__ void refresh_shared_chr(bool valid) {
        if (!S.chr_shared || C.chr) return;
        u32 pend = __ballot_sync(0xFFFFFFFFu, valid && rw(R_CHRD) != 0u);
        while (pend) {
            const u32 L = __ffs(pend) - 1;
            pend &= pend - 1;
            const u32 eL = __shfl_sync(0xFFFFFFFFu, e, L);
            const uint4* cv = reinterpret_cast<const uint4*>(S.chr_ram + static_cast<u64>(eL) * kChrRamBytes);
            uint4* dc = reinterpret_cast<uint4*>(S.chr_shared + static_cast<u64>(eL) * kChrRamBytes);
#pragma unroll 4
            for (u32 i = lane; i < kChrRamBytes / 16; i += 32) dc[i] = cv[i];
        }
        __syncwarp();
        if (valid) ww(R_CHRD, 0u);
    }

    __device__ __forceinline__ void snapshot_frozen() {
        u32 pend = __ballot_sync(0xFFFFFFFFu, froze != 0);
        while (pend) {
            const u32 L = __ffs(pend) - 1;
            pend &= pend - 1;
            const u32 eL = __shfl_sync(0xFFFFFFFFu, e, L);
            const u32 sL = __shfl_sync(0xFFFFFFFFu, slot, L);
            const u64 sl = static_cast<u64>(eL) * 4 + sL;
            const uint4* ntv = reinterpret_cast<const uint4*>(S.nt + static_cast<u64>(eL) * kNtBytes);
            uint4* dnt = reinterpret_cast<uint4*>(S.snap_nt + sl * kNtBytes);
            const uint4 q0 = ntv[lane], q1 = ntv[lane + 32], q2 = ntv[lane + 64], q3 = ntv[lane + 96];
            u32* doam = reinterpret_cast<u32*>(S.snap_oam + sl * kOamBytes);
            const u32 o0 = sh.oam[lane][L], o1 = sh.oam[lane + 32][L];
            dnt[lane] = q0; dnt[lane + 32] = q1; dnt[lane + 64] = q2; dnt[lane + 96] = q3;
            doam[lane] = o0; doam[lane + 32] = o1;
            if (S.snap_chr && !C.chr) {
                // no CHR-RAM write since the shared snapshot: the slot points at it, else it takes its own copy
                const bool shared = S.chr_shared && sh.regs[R_CHRD][L] == 0u;
                if (lane == 0 && S.chr_ref) S.chr_ref[sl] = shared ? 1u : 0u;
                if (!shared) {
                    const uint4* cv = reinterpret_cast<const uint4*>(S.chr_ram + static_cast<u64>(eL) * kChrRamBytes);
                    uint4* dc = reinterpret_cast<uint4*>(S.snap_chr + sl * kChrRamBytes);
#pragma unroll 4
                    for (u32 i = lane; i < kChrRamBytes / 16; i += 32) dc[i] = cv[i];
                }
            }
        }
        froze = 0;
    }

    __device__ __forceinline__ Hit0 sprite0_eval() const;
    __device__ __forceinline__ void mmc2_resolve();

    // -------- PPU settle (patch:2114-2240)
    __device__ __forceinline__ u32 dots_to_event() const {
        const u32 cur = frame_dot;
        const u32 skip = (log_ctl & kLcShort) ? 1u : 0u;
        const u32 fd = kFrameDots - skip;
        auto dist = [&](u32 ev) { return ev > cur ? ev - cur : fd - cur + ev; };
        u32 next = fd - cur;
        next = min(next, dist(kVblankFlagDot));
        next = min(next, dist(kVblankDot));
        next = min(next, dist(kStatusClearDot));
        next = min(next, dist(kPreRenderDot));
        const u32 s0 = rw(R_S0) & kS0DotMask;
        if (s0 != 0) next = min(next, dist(s0));
        if constexpr (BOARD == kMmc3) {
            // Only the scanline-counter clock that raises the IRQ is an event: the clocks before it change the
            // counter alone and settle applies them in one pass. Nothing changes what they do but a store to
            // $2000 / $2001 or to the IRQ registers, and those settle first and reschedule (step6502).
            if ((mask & 0x18u) != 0 && (ctrl & 0x38u) != 0x18u && mreg(13) != 0) {
                const u32 c = mreg(12), lat = mreg(11);
                const u32 c1 = (c == 0 || mreg(14) != 0) ? lat : c - 1;   // the counter after the next clock
                const u32 line = cur / kDots, dot = cur % kDots;
                // this frame's clocks: index 0..239 the visible lines, 240 the pre-render line; i0 = the next one
                const u32 i0 = line < 240 ? line + (dot >= kMmc3VisibleClock ? 1u : 0u)
                                          : (line < 261 || dot < kMmc3PreClock) ? 240u : 241u;
                const u32 i = i0 + c1;   // the (c1 + 1)-th clock from here leaves the counter at 0
                if (i <= 240) {
                    const u32 t = i < 240 ? i * kDots + kMmc3VisibleClock : 261u * kDots + kMmc3PreClock;
                    next = min(next, t - cur);
                }
            }
        }
        return next;
    }

    __device__ __forceinline__ void mmc3_clock() {
        u32 cnt = mreg(12), latch = mreg(11), reload = mreg(14);
        if (cnt == 0 || reload) { cnt = latch; set_mreg(14, 0); }
        else --cnt;
        set_mreg(12, cnt);
        if (cnt == 0 && mreg(13)) set_field(R_IO, 24, 0xFF, 1);
    }

    __device__ __forceinline__ void settle(u32 dots) {
        const u32 start = frame_dot;
        u32 end = start + dots;
        if ((log_ctl & kLcShort) && end >= kFrameDots - 1) end += 1;
        const u32 frames = end / kFrameDots;
        for (u32 fo = 0; fo <= frames; ++fo) {
            const u32 base = fo * kFrameDots;
            auto crossed = [&](u32 ev) { const u32 t = base + ev; return t > start && t <= end; };
            const u32 sched = rw(R_S0);
            const u32 s0 = sched & kS0DotMask;
            if (s0 != 0 && crossed(s0)) {
                const bool known = (sched & kS0Known) && ((sched >> 20) & 0x1FFu) == log_n;
                const Hit0 found = known ? Hit0{s0, (sched & kS0Hit) != 0} : sprite0_eval();
                const bool reached = base + found.dot <= end;
                if (found.hit && reached) status |= 0x40u;
                ww(R_S0, found.dot != 0 && !reached
                             ? (found.dot | kS0Evaluate | kS0Known | (found.hit ? kS0Hit : 0u) | (log_n << 20))
                             : 0u);
            }
            if (crossed(kVblankFlagDot)) status |= 0x80u;
            if (crossed(kVblankDot)) {
                if (ctrl & 0x80u) nmi = 1;
                log_freeze();
            }
            if (crossed(kStatusClearDot)) status &= 0x1Fu;
            if (crossed(kPreRenderDot)) {
                status &= 0x1Fu;
                log_capture();
                const u32 y0 = oam_rd(0);
                ww(R_S0, y0 < 239u ? (nesle_dot(static_cast<int>(y0 + 1) * 341 - 20) | kS0Evaluate) : 0u);
            }
        }
        if constexpr (BOARD == kMmc3) {
            if ((mask & 0x18u) != 0 && (ctrl & 0x38u) != 0x18u) {
                for (u32 la = start / kDots; la <= end / kDots; ++la) {
                    const u32 line = la % kLines;
                    const u32 cd = line < 240 ? kMmc3VisibleClock : line == 261 ? kMmc3PreClock : 0xFFFFFFFFu;
                    if (cd == 0xFFFFFFFFu) continue;
                    const u32 t = la * kDots + cd;
                    if (t > start && t <= end) mmc3_clock();
                }
            }
        }
        frame_dot = end % kFrameDots;
        frame += frames;
        if (frames) log_ctl &= ~kLcShort;
    }

    // -------- CPU bus
    __device__ __forceinline__ u32 rd_io(u32 addr) {
        if (addr < 0x4000u) {
            switch (addr & 7u) {
                case 2: {
                    const u32 ob = rw(R_PPU1) >> 24;
                    const u32 v = (status & 0xE0u) | (ob & 0x1Fu);
                    status &= 0x7Fu;
                    set_field(R_PPU1, 16, 0xFF, 0);
                    return v;
                }
                case 4: return oam_rd(oam_addr);
                case 7: {
                    u32 vt = rw(R_VT);
                    const u32 v16 = vt & 0xFFFFu;
                    const u32 pa = v16 & 0x3FFFu;
                    u32 value;
                    u32 rb = rw(R_PPU2) & 0xFFu;
                    if (pa >= 0x3F00u) {
                        value = ppu_mem_rd(pa);
                        rb = ppu_mem_rd(pa - 0x1000u);
                    } else {
                        value = rb;
                        ppu_address(pa);   // the buffer refills through the bank the address picks
                        rb = ppu_mem_rd(pa);
                    }
                    set_field(R_PPU2, 0, 0xFF, rb);
                    const u32 nv = (v16 + ((ctrl & 4u) ? 32u : 1u)) & 0x7FFFu;
                    ww(R_VT, (vt & 0xFFFF0000u) | nv);
                    log_event(kEvDataRead, 0, 0);
                    ppu_address(nv & 0x3FFFu);
                    set_field(R_PPU1, 24, 0xFF, value);
                    return value;
                }
                default: return 0;
            }
        }
        if (addr == 0x4015u) return (rw(R_DMC_A) & 0xFFFFu) ? 0x10u : 0u;
        if (addr == 0x4016u) {
            const u32 io = rw(R_IO);
            const u32 shift = io & 0xFF, count = (io >> 8) & 0xFF, strobe = (io >> 16) & 0xFF;
            u32 bit;
            if (strobe) bit = pad & 1u;
            else if (count < 8) { bit = (shift >> count) & 1u; set_field(R_IO, 8, 0xFF, count + 1); }
            else bit = 1u;
            return 0x40u | bit;
        }
        if (addr == 0x4017u) return 0x40u;
        if (addr < 0x6000u) return (addr >> 8) & 0xFFu;
        if (addr < 0x8000u) {
            if constexpr (BOARD == kMmc1) { if (mreg(3) & 0x10u) return (addr >> 8) & 0xFFu; }
            return prgram8()[prgram_index(addr - 0x6000u)];
        }
        return prg_rd(addr);
    }

    __device__ __forceinline__ u32 rd(u32 addr) {
        if (addr < 0x2000u) return ram_rd(addr);
        if (addr >= 0x8000u) return prg_rd(addr);
        return rd_io(addr);
    }

    __device__ __forceinline__ void mmc1_sync() {
        const u32 ctl = mreg(0), offs = mreg(1) & 0x10u, prg = mreg(3);
        auto prg8 = [&](u32 s, u32 b) { ww(R_PRGPG + s, (b & C.prg_page_mask) << 13); };
        auto prg16 = [&](u32 s, u32 b) { prg8(2 * s, 2 * b); prg8(2 * s + 1, 2 * b + 1); };
        auto chr4 = [&](u32 s, u32 b) { for (u32 i = 0; i < 4; ++i) ww(R_CHRPG + 4 * s + i, ((4 * b + i) & C.chr_page_mask) << 10); };
        if ((ctl & 0x0Cu) == 0x0Cu) { prg16(0, prg + offs); prg16(1, 0x0Fu + offs); }
        else if ((ctl & 0x0Cu) == 0x08u) { prg16(1, prg + offs); prg16(0, offs); }
        else { prg16(0, (prg & ~1u) + offs); prg16(1, (prg & ~1u) + offs + 1u); }
        if (ctl & 0x10u) { chr4(0, mreg(1)); chr4(1, mreg(2)); }
        else { chr4(0, mreg(1) & 0xFEu); chr4(1, mreg(1) | 1u); }
        if (C.arrangement != 2) {
            const u32 mm = ctl & 3u;
            const u32 map = mm == 0 ? kPageSingleLow : mm == 1 ? kPageSingleHigh : mm == 2 ? kPageVertical : kPageHorizontal;
            set_field(R_PPU2, 24, 0xFF, map);
        }
    }
    __device__ __forceinline__ void mmc3_sync() {
        const u32 sel = mreg(8), r6 = mreg(6) & 0x7Fu;
        auto prg8 = [&](u32 s, u32 b) { ww(R_PRGPG + s, (b & C.prg_page_mask) << 13); };
        auto chr1 = [&](u32 s, u32 b) { ww(R_CHRPG + s, (b & C.chr_page_mask) << 10); };
        if (sel & 0x40u) { prg8(2, r6); prg8(0, 0x7E); } else { prg8(0, r6); prg8(2, 0x7E); }
        prg8(1, mreg(7) & 0x7Fu);
        prg8(3, 0x7F);
        const u32 f = (sel & 0x80u) ? 4u : 0u;
        chr1(0 ^ f, mreg(0) & 0xFEu); chr1(1 ^ f, mreg(0) | 1u);
        chr1(2 ^ f, mreg(1) & 0xFEu); chr1(3 ^ f, mreg(1) | 1u);
        chr1(4 ^ f, mreg(2)); chr1(5 ^ f, mreg(3)); chr1(6 ^ f, mreg(4)); chr1(7 ^ f, mreg(5));
        if (C.arrangement != 2) set_field(R_PPU2, 24, 0xFF, (mreg(9) & 1u) ? kPageHorizontal : kPageVertical);
    }

    // CNROM (patch:2982-2990 paged::sync): PRG 8 KB pages 0-3 (a 16 KB image mirrors through the mask), CHR 1 KB
    // pages of the 8 KB bank in register 0.
    __device__ __forceinline__ void cnrom_sync() {
        for (u32 s = 0; s < 4; ++s) ww(R_PRGPG + s, (s & C.prg_page_mask) << 13);
        for (u32 s = 0; s < 8; ++s) ww(R_CHRPG + s, ((mreg(0) * 8u + s) & C.chr_page_mask) << 10);
    }

    // MMC2 (patch:3027-3035 paged::sync): the switchable 8 KB page at $8000 and the last three; each 4 KB CHR half
    // from the register its latch picks ($FD: 0 / 2, $FE: 1 / 3); register 5 set = vertical mirroring.
    __device__ __forceinline__ void mmc2_chr4(u32 half) {
        const u32 b = mreg(2u * half + (mreg(6u + half) & 1u));
        for (u32 i = 0; i < 4; ++i) ww(R_CHRPG + 4 * half + i, ((4 * b + i) & C.chr_page_mask) << 10);
    }
    __device__ __forceinline__ void mmc2_sync() {
        auto prg8 = [&](u32 s, u32 b) { ww(R_PRGPG + s, (b & C.prg_page_mask) << 13); };
        prg8(0, mreg(4)); prg8(1, ~2u); prg8(2, ~1u); prg8(3, ~0u);
        mmc2_chr4(0);
        mmc2_chr4(1);
        if (C.arrangement != 2) set_field(R_PPU2, 24, 0xFF, mreg(5) ? kPageVertical : kPageHorizontal);
    }
    // The VRAM address the CPU puts on the PPU bus ($2006 / $2007): MMC2's latch hook ($0FD0-$0FEF / $1FD0-$1FEF,
    // patch:3195-3222), the change logged while a frame is drawn (patch:615-636 bus_ppu_address).
    __device__ __forceinline__ void ppu_address(u32 addr) {
        if constexpr (BOARD == kMmc2) {
            const u32 high = (addr >> 8) & 0x3Fu, low = addr & 0xF0u;
            if (high >= 0x20u || (high & 0x0Fu) != 0x0Fu || (low != 0xD0u && low != 0xE0u)) return;
            const u32 half = high >> 4, latch = low == 0xE0u ? 1u : 0u;
            const u32 before = mreg(6u + half);
            set_mreg(6u + half, latch);
            mmc2_chr4(half);
            if (before != latch) log_event(kEvMmc2, latch, 6u + half);
        } else {
            (void)addr;
        }
    }

    __device__ __forceinline__ void board_write(u32 addr, u32 v) {
        if constexpr (BOARD == kCnrom) {
            (void)addr;   // the bank latch (no bus conflicts: an iNES 1.0 image declares none)
            set_mreg(0, v);
            cnrom_sync();
        } else if constexpr (BOARD == kMmc1) {
            if (v & 0x80u) { set_mreg(0, mreg(0) | 0x0Cu); set_mreg(4, 0); set_mreg(5, 0); mmc1_sync(); return; }
            const u32 cnt = mreg(5);
            const u32 sh = mreg(4) | ((v & 1u) << cnt);
            if (cnt + 1 < 5) { set_mreg(4, sh); set_mreg(5, cnt + 1); return; }
            set_mreg((addr >> 13) - 4u, sh);
            set_mreg(4, 0);
            set_mreg(5, 0);
            mmc1_sync();
        } else if constexpr (BOARD == kMmc3) {
            switch (addr & 0xE001u) {
                case 0x8000u: set_mreg(8, v); break;
                case 0x8001u: set_mreg(mreg(8) & 7u, v); break;
                case 0xA000u: set_mreg(9, v); break;
                case 0xA001u: set_mreg(10, v); return;
                case 0xC000u: set_mreg(11, v); return;
                case 0xC001u: set_mreg(14, 1); return;
                case 0xE000u: set_mreg(13, 0); set_field(R_IO, 24, 0xFF, 0); return;
                default: set_mreg(13, 1); return;
            }
            mmc3_sync();
        } else if constexpr (BOARD == kMmc2) {   // patch:3147-3156
            switch (addr & 0xF000u) {
                case 0xA000u: set_mreg(4, v & 0x0Fu); break;
                case 0xB000u: set_mreg(0, v & 0x1Fu); break;
                case 0xC000u: set_mreg(1, v & 0x1Fu); break;
                case 0xD000u: set_mreg(2, v & 0x1Fu); break;
                case 0xE000u: set_mreg(3, v & 0x1Fu); break;
                case 0xF000u: set_mreg(5, (v & 1u) ^ 1u); break;
                default: return;   // $8000-$9FFF: no register
            }
            mmc2_sync();
        }
    }

    __device__ __forceinline__ void mapper_write(u32 addr, u32 v) {
        if constexpr (BOARD == kUxrom) {
            prg_bank = v & C.bank_mask;
        } else if constexpr (board_paged(BOARD)) {
            if (log_active()) {
                u32 before[8];
                for (int i = 0; i < 8; ++i) before[i] = rw(R_CHRPG + i);
                const u32 mir = mirroring();
                const u32 creg = rw(R_MREG);   // registers 0-3 (MMC2's CHR registers)
                board_write(addr, v);
                for (u32 i = 0; i < 8; ++i) {
                    const u32 pg = rw(R_CHRPG + i);
                    if (pg != before[i]) log_event(kEvChr, pg >> 10, i);
                }
                if (mirroring() != mir) log_event(kEvMirror, mirroring(), 0);
                if constexpr (BOARD == kMmc2) {   // the CHR registers the write changed (patch:661-665)
                    const u32 now_c = rw(R_MREG);
                    for (u32 i = 0; i < 4; ++i)
                        if (((now_c ^ creg) >> (8 * i)) & 0xFFu) log_event(kEvMmc2, (now_c >> (8 * i)) & 0xFFu, i);
                }
            } else {
                board_write(addr, v);
            }
        }
    }

    __device__ __forceinline__ void wr_io(u32 addr, u32 v) {
        if (addr < 0x4000u) {
            switch (addr & 7u) {
                case 0: {
                    ctrl = v;
                    const u32 vt = rw(R_VT);
                    const u32 t = ((vt >> 16) & 0xF3FFu) | ((v & 3u) << 10);
                    ww(R_VT, (vt & 0xFFFFu) | (t << 16));
                    log_event(kEvCtrl, v, 0);
                    break;
                }
                case 1: mask = v; log_event(kEvMask, v, 0); break;
                case 3: oam_addr = v; break;
                case 4: oam_wr(oam_addr, v); oam_addr = (oam_addr + 1) & 0xFFu; break;
                case 5: {
                    const u32 p1 = rw(R_PPU1);
                    const u32 w = (p1 >> 16) & 0xFFu;
                    log_event(kEvScroll, v, w);
                    const u32 vt = rw(R_VT);
                    u32 t = vt >> 16;
                    if (w == 0) {
                        t = (t & 0xFFE0u) | (v >> 3);
                        ww(R_PPU1, (p1 & 0xFF0000FFu) | ((v & 7u) << 8) | (1u << 16));
                        set_field(R_LOGN, 16, 0xFF, v);
                    } else {
                        t = (t & 0x8C1Fu) | ((v & 0xF8u) << 2) | ((v & 7u) << 12);
                        ww(R_PPU1, p1 & 0xFF00FFFFu);
                        set_field(R_LOGN, 24, 0xFF, v);
                    }
                    ww(R_VT, (vt & 0xFFFFu) | (t << 16));
                    break;
                }
                case 6: {
                    const u32 p1 = rw(R_PPU1);
                    const u32 w = (p1 >> 16) & 0xFFu;
                    log_event(kEvAddr, v, w);
                    const u32 vt = rw(R_VT);
                    u32 t = vt >> 16, vv = vt & 0xFFFFu;
                    if (w == 0) {
                        t = (t & 0x00FFu) | ((v & 0x3Fu) << 8);
                        ww(R_PPU1, (p1 & 0xFF00FFFFu) | (1u << 16));
                    } else {
                        t = (t & 0x7F00u) | v;
                        vv = t;
                        ww(R_PPU1, p1 & 0xFF00FFFFu);
                    }
                    ww(R_VT, vv | (t << 16));
                    if (w != 0) ppu_address(vv);
                    break;
                }
                case 7: {
                    const u32 vt = rw(R_VT);
                    const u32 v16 = vt & 0xFFFFu;
                    const u32 pa = v16 & 0x3FFFu;
                    ppu_mem_wr(v16, v);
                    if (pa >= 0x3F00u) log_event(kEvPalette, v, pal_index(pa));
                    else log_event(kEvDataWrite, 0, 0);
                    const u32 nv = (v16 + ((ctrl & 4u) ? 32u : 1u)) & 0x7FFFu;
                    ww(R_VT, (vt & 0xFFFF0000u) | nv);
                    ppu_address(nv & 0x3FFFu);
                    break;
                }
                default: break;
            }
            set_field(R_PPU1, 24, 0xFF, v);
            return;
        }
        if (addr == 0x4014u) {
            // OAM DMA: 256 bytes from page v; a RAM page into OAM from address 0 is copied as words
            if (v < 0x20u && oam_addr == 0) {
                const u32 base = ((v & 7u) << 8) >> 2;
#pragma unroll 8
                for (u32 i = 0; i < 64; ++i) sh.oam[i][lane] = sh.ram[base + i][lane];
            } else {
                for (u32 i = 0; i < 256; ++i) oam_wr((oam_addr + i) & 0xFFu, rd((v << 8) + i));
            }
            dma = 1;
            return;
        }
        if (addr == 0x4016u) {
            const u32 strobe = v & 1u;
            if (strobe) ww(R_IO, (rw(R_IO) & 0xFF000000u) | pad | (1u << 16));
            else set_field(R_IO, 16, 0xFF, 0);
            return;
        }
        if (addr == 0x4010u || addr == 0x4013u || addr == 0x4015u) {
            u32 da = rw(R_DMC_A);
            u32 bytes_left = da & 0xFFFFu, control = (da >> 16) & 0xFF, length = da >> 24;
            if (addr == 0x4010u) control = v;
            else if (addr == 0x4013u) length = v;
            else if (!(v & 0x10u)) bytes_left = 0;
            else if (bytes_left == 0) bytes_left = length * 16u + 1u;
            ww(R_DMC_A, bytes_left | (control << 16) | (length << 24));
            ww(R_DMC_EV, 0); ww(R_DMC_EV + 1, 0);
            dmc_at = 0;
            return;
        }
        if (addr < 0x6000u) return;
        if (addr < 0x8000u) {
            if constexpr (BOARD == kMmc1) { if (mreg(3) & 0x10u) return; }
            prgram8()[prgram_index(addr - 0x6000u)] = static_cast<u8>(v);
            return;
        }
        mapper_write(addr, v);
    }

    __device__ __forceinline__ void wr(u32 addr, u32 v) {
        if (addr < 0x2000u) { ram_wr(addr, v); return; }
        wr_io(addr, v);
    }

    // -------- DMC (patch:480-547)
    __device__ __forceinline__ u32 dmc_service(u64 nowc, bool steal) {
        u64 be = rw(R_DMC_END) | (static_cast<u64>(rw(R_DMC_END + 1)) << 32);
        const u32 da = rw(R_DMC_A), db = rw(R_DMC_B);
        u32 bytes_left = da & 0xFFFFu, control = (da >> 16) & 0xFF, length = da >> 24;
        u32 rate = db & 0xFF, full = (db >> 8) & 0xFF;
        const u64 byte_cycles = 8ull * dmc_period(rate);
        auto skip = [&] { if (be <= nowc) be += ((nowc - be) / byte_cycles + 1) * byte_cycles; };
        u32 stolen = 0;
        if (!full) skip();
        for (;;) {
            if (full) {
                if (be > nowc) break;
                full = 0;
                be += byte_cycles;
                if (bytes_left == 0) { skip(); break; }
            }
            if (bytes_left == 0) break;
            full = 1;
            if (--bytes_left == 0 && (control & 0x40u)) bytes_left = length * 16u + 1u;
            if (steal) { stolen += 4; nowc += 4; }
        }
        const u32 nr = control & 0x0Fu;
        if (nr != rate) {
            const u64 oldp = dmc_period(rate);
            const u64 later = (be - nowc - 1) / oldp;
            be = be - later * oldp + later * dmc_period(nr);
            rate = nr;
        }
        ww(R_DMC_END, static_cast<u32>(be)); ww(R_DMC_END + 1, static_cast<u32>(be >> 32));
        ww(R_DMC_A, bytes_left | (control << 16) | (length << 24));
        ww(R_DMC_B, rate | (full << 8));
        const u64 ev = full ? be : kDmcIdle;
        ww(R_DMC_EV, static_cast<u32>(ev)); ww(R_DMC_EV + 1, static_cast<u32>(ev >> 32));
        dmc_at = ev;
        return stolen;
    }
    __device__ __forceinline__ u64 dmc_event() const { return dmc_at; }

    // -------- 6502
    __device__ __forceinline__ void push(u32 v) { ram_wr(0x100u | sp, v); sp = (sp - 1) & 0xFFu; }
    __device__ __forceinline__ u32 pull() { sp = (sp + 1) & 0xFFu; return ram_rd(0x100u | sp); }
    __device__ __forceinline__ void nz(u32 v) { p = (p & ~(FZ | FN)) | (v == 0 ? FZ : 0u) | (v & 0x80u); }
    __device__ __forceinline__ u32 fetch(u32 addr) { return addr >= 0x8000u ? prg_rd(addr) : rd(addr); }

    __device__ __forceinline__ void interrupt(u32 vector) {
        push(pc >> 8);
        push(pc & 0xFFu);
        push((p & ~FB) | FU);
        p |= FI;
        pc = fetch(vector) | (fetch(vector + 1) << 8);
        cycles += 7;
    }

    struct Step { u32 cycles, opcode, pc; bool illegal; };

    __device__ __forceinline__ Step step6502() {
        const u32 pc0 = pc;
        // opcode and both operand bytes fetched together (PRG: three independent loads)
        u32 op, b1, b2;
        if (pc0 >= 0x8000u && pc0 <= 0xFFFDu) {
            op = prg_rd(pc0); b1 = prg_rd(pc0 + 1); b2 = prg_rd(pc0 + 2);
        } else {
            op = fetch(pc0); b1 = 0; b2 = 0;
        }
        const u32 d = dtab[op];
        const u32 mode = d & 15u, opn = (d >> 4) & 63u;
        u32 cyc = (d >> 10) & 15u;
        if (opn == O_ILL) return Step{0, op, pc0, true};
        if (pc0 < 0x8000u || pc0 > 0xFFFDu) {
            if (mode >= M_IMM) b1 = fetch((pc0 + 1) & 0xFFFFu);
            if (mode >= M_ABS && mode <= M_IND) b2 = fetch((pc0 + 2) & 0xFFFFu);
        }
        // ---- operand / effective address: selects from the decode entry's recipe (no branch but the rare
        // indirect modes), the operand bytes fetched speculatively above
        u32 val = 0;
        pc = (pc0 + 1u + ((d >> kDLen) & 3u)) & 0xFFFFu;
        const u32 idx = (d & kDX) ? x : ((d & kDY) ? y : 0u);
        u32 base = (d & kDAbs) ? (b1 | (b2 << 8)) : b1;
        if (d & kDInd) {   // (zp,X): pointer at zp b1 + X; (zp),Y: pointer at zp b1, + Y; JMP (ind): the operand
            if (mode != M_IND) {
                const u32 z = (d & kDX) ? ((b1 + x) & 0xFFu) : b1;
                base = ram_rd(z) | (ram_rd((z + 1) & 0xFFu) << 8);
            }
        }
        u32 ea = (base + ((d & kDInd) && (d & kDX) ? 0u : idx)) & ((d & kDZp) ? 0xFFu : 0xFFFFu);
        const bool cross = ((base ^ ea) & 0xFF00u) != 0;
        if ((d >> 14) & cross) ++cyc;
        // operand value for the reading operations
        const bool reads = (opn >= O_LDA && opn <= O_LDY) || (opn >= O_ADC && opn <= O_DEC);
        if (reads) val = mode == M_IMM ? b1 : mode == M_ACC ? a : rd(ea);
        bool store = false;   // one store site for STA / STX / STY and read-modify-write results
        u32 wv = 0;
        // ---- operation
        switch (opn) {
            case O_LDA: a = val; nz(a); break;
            case O_LDX: x = val; nz(x); break;
            case O_LDY: y = val; nz(y); break;
            case O_STA: store = true; wv = a; break;
            case O_STX: store = true; wv = x; break;
            case O_STY: store = true; wv = y; break;
            case O_SBC: val ^= 0xFFu; [[fallthrough]];
            case O_ADC: {
                const u32 s = a + val + (p & FC);
                p = (p & ~(FC | FV)) | (s > 0xFFu ? FC : 0u) | ((~(a ^ val) & (a ^ s) & 0x80u) ? FV : 0u);
                a = s & 0xFFu;
                nz(a);
                break;
            }
            case O_AND: a &= val; nz(a); break;
            case O_ORA: a |= val; nz(a); break;
            case O_EOR: a ^= val; nz(a); break;
            case O_CMP: case O_CPX: case O_CPY: {
                const u32 r = opn == O_CMP ? a : opn == O_CPX ? x : y;
                p = (p & ~FC) | (r >= val ? FC : 0u);
                nz((r - val) & 0xFFu);
                break;
            }
            case O_BIT: p = (p & ~(FZ | FV | FN)) | ((a & val) == 0 ? FZ : 0u) | (val & 0xC0u); break;
            case O_ASL: case O_LSR: case O_ROL: case O_ROR: case O_INC: case O_DEC: {
                u32 r;
                const u32 cin = p & FC;
                switch (opn) {
                    case O_ASL: p = (p & ~FC) | (val >> 7); r = (val << 1) & 0xFFu; break;
                    case O_ROL: p = (p & ~FC) | (val >> 7); r = ((val << 1) | cin) & 0xFFu; break;
                    case O_LSR: p = (p & ~FC) | (val & 1u); r = val >> 1; break;
                    case O_ROR: p = (p & ~FC) | (val & 1u); r = (val >> 1) | (cin << 7); break;
                    case O_INC: r = (val + 1) & 0xFFu; break;
                    default: r = (val - 1) & 0xFFu; break;
                }
                nz(r);
                if (mode == M_ACC) a = r; else { store = true; wv = r; }
                break;
            }
            case O_INX: x = (x + 1) & 0xFFu; nz(x); break;
            case O_INY: y = (y + 1) & 0xFFu; nz(y); break;
            case O_DEX: x = (x - 1) & 0xFFu; nz(x); break;
            case O_DEY: y = (y - 1) & 0xFFu; nz(y); break;
            case O_TAX: x = a; nz(x); break;
            case O_TAY: y = a; nz(y); break;
            case O_TXA: a = x; nz(a); break;
            case O_TYA: a = y; nz(a); break;
            case O_TSX: x = sp; nz(x); break;
            case O_TXS: sp = x; break;
            case O_CLC: p &= ~FC; break;
            case O_SEC: p |= FC; break;
            case O_CLI: p &= ~FI; break;
            case O_SEI: p |= FI; break;
            case O_CLV: p &= ~FV; break;
            case O_CLD: p &= ~FD; break;
            case O_SED: p |= FD; break;
            case O_NOP: break;
            case O_PHA: push(a); break;
            case O_PHP: push(p | FB | FU); break;
            case O_PLA: a = pull(); nz(a); break;
            case O_PLP: p = (pull() & ~FB) | FU; break;
            case O_JMP:
                if (mode == M_ABS) pc = ea;
                else pc = rd(ea) | (rd((ea & 0xFF00u) | ((ea + 1) & 0xFFu)) << 8);
                break;
            case O_JSR: {
                const u32 ret = (pc0 + 2) & 0xFFFFu;
                push(ret >> 8);
                push(ret & 0xFFu);
                pc = ea;
                break;
            }
            case O_RTS: { const u32 lo = pull(); const u32 hi = pull(); pc = (((hi << 8) | lo) + 1) & 0xFFFFu; break; }
            case O_RTI: {
                p = (pull() & ~FB) | FU;
                const u32 lo = pull(); const u32 hi = pull();
                pc = (hi << 8) | lo;
                break;
            }
            case O_BRK: {
                const u32 ret = (pc0 + 2) & 0xFFFFu;
                push(ret >> 8);
                push(ret & 0xFFu);
                push(p | FB | FU);
                p |= FI;
                pc = fetch(0xFFFEu) | (fetch(0xFFFFu) << 8);
                break;
            }
            default: {   // branches: O_BPL.. O_BEQ in (flag, value) pairs
                const u32 k = opn - O_BPL;
                const u32 flag = k < 2 ? FN : k < 4 ? FV : k < 6 ? FC : FZ;
                const bool want = (k & 1u) != 0;
                if (((p & flag) != 0) == want) {
                    const u32 to = (pc + static_cast<u32>(static_cast<int>(static_cast<int8_t>(b1)))) & 0xFFFFu;
                    cyc += ((to ^ pc) & 0xFF00u) ? 2u : 1u;
                    pc = to;
                }
                break;
            }
        }
        if constexpr (BOARD == kMmc3) {
            // $2000 / $2001 (and mirrors) or the IRQ registers: the counter's clocks up to this instruction run
            // under the old values first, exactly as when every clock was its own event
            if (store && ((ea & 0xE006u) == 0x2000u || ea >= 0xC000u)) {
                if (pend != 0) { settle(pend); pend = 0; }
                resched = 1;
            }
        }
        if (store) wr(ea, wv);
        cycles += cyc;
        return Step{cyc, op, pc0, false};
    }

    // One instruction with NMI / IRQ entry, frame-log stamps, DMA stall and DMC steals (patch:834-861).
    __device__ __forceinline__ Step console_step(u32& ppu_cycles) {
        const u32 pending = pend;
        const u64 before = cycles;
        if (nmi) {
            nmi = 0;
            interrupt(0xFFFAu);
        } else if constexpr (BOARD == kMmc3) {
            if ((rw(R_IO) >> 24) && !(p & FI)) interrupt(0xFFFEu);
        }
        now = frame_dot + pending + static_cast<u32>(cycles - before) * 3u;
        const u32 logged = log_n;
        const Step s = step6502();
        if (s.illegal) { ppu_cycles = 0; return s; }
        // the rare work after an instruction (frame-log cycle stamps, OAM DMA, a DMC fetch) behind one branch
        if ((log_n != logged) | (dma != 0u) | (cycles >= dmc_event())) {
            if (log_n != logged) {
                u32* bank = writing_bank();
                const u32 c = (s.cycles > 15u ? 15u : s.cycles) << 17;
                for (u32 i = logged; i < log_n && i < kLogEv; ++i) bank[kLogHdr + 2 * i] |= c;
            }
            if (dma) { dma = 0; cycles += 513u + static_cast<u32>(cycles & 1u); }
            if (cycles >= dmc_event()) cycles += dmc_service(cycles, true);
        }
        ppu_cycles = static_cast<u32>(cycles - before) * 3u;
        return s;
    }

    // Dots from frame_dot to the next scanline-counter clock (the reference's batch_ppu_dots_until_scanline_clock,
    // patch:1881-1902 and its short-frame use, patch:2061-2064).
    __device__ __forceinline__ u32 dots_to_counter_clock() const {
        const u32 cur = frame_dot, line = cur / kDots, dot = cur % kDots;
        u32 d;
        if (line < 240u) {
            d = dot < kMmc3VisibleClock ? kMmc3VisibleClock - dot
              : line + 1u < 240u ? kDots - dot + kMmc3VisibleClock : (261u - line) * kDots + kMmc3PreClock - dot;
        } else if (line < 261u) {
            d = (261u - line) * kDots + kMmc3PreClock - dot;
        } else {
            d = dot < kMmc3PreClock ? kMmc3PreClock - dot : kDots - dot + kMmc3VisibleClock;
        }
        if ((log_ctl & kLcShort) && cur + d >= kFrameDots) d -= 1u;
        return d;
    }

    __device__ __forceinline__ void fast_forward() {
        if (nmi) return;
        u32 to = dots_to_event();
        if constexpr (BOARD == kMmc3) {
            // The reference schedules every counter clock as an event, so a skip ends at the next clock. Only the clock
            // that raises the IRQ is an event here; that is the same wherever no IRQ can be taken, but an IRQ the
            // settle before this skip raised (the jump crossed its clock) is taken after the next clock, not after the
            // next other event.
            if ((rw(R_IO) >> 24) && !(p & FI)) to = min(to, dots_to_counter_clock());
        }
        const u32 jumps = (to + 8u) / 9u;
        if (jumps == 0) return;
        const u32 cc = jumps * 3u;
        cycles += cc;
        if (cycles >= dmc_event()) (void)dmc_service(cycles, false);
        settle(cc * 3u);
    }

    // Run to absolute PPU dot `target` (rl/csrc/nes_machine.cuh:67-103). Returns pc << 8 | opcode on a fault.
    // Called by all 32 lanes of the warp together (`run` false for lanes with nothing to emulate). Lanes drift to
    // different 6502 addresses after a divergent branch; each loop turn only the lanes at the lowest program counter
    // execute, so lanes that skipped a block wait for the others and the warp runs one instruction body per turn.
    // Every lane's own state advances exactly as in the sequential loop.
    __device__ __forceinline__ u32 step_until(u64 target, bool run) {
        u32 fault = 0;
        pend = 0;
        resched = 0;
        u32 to_event = run ? dots_to_event() : 0u;
        u32 instructions = 0;
        bool going = run;
        while (__any_sync(0xFFFFFFFFu, going)) {
            const u32 lead = __reduce_min_sync(0xFFFFFFFFu, going ? pc : 0x10000u);
            if (!going || pc != lead) continue;
            if (instructions >= kBudget) { going = false; continue; }
            if (pend >= to_event) {
                settle(pend);
                pend = 0;
                to_event = dots_to_event();
                if (frame * kFrameDots + frame_dot >= target) { going = false; continue; }
            }
            u32 pc_cycles;
            const Step st = console_step(pc_cycles);
            if (st.illegal) { fault = (st.pc << 8) | st.opcode; going = false; continue; }
            pend += pc_cycles;
            ++instructions;
            if constexpr (BOARD == kMmc3) {
                if (resched) { resched = 0; to_event = dots_to_event(); }   // from the settled frame_dot
            }
            if (st.opcode == 0x4Cu && pc == st.pc) {
                settle(pend);
                pend = 0;
                if (frame * kFrameDots + frame_dot >= target) { going = false; continue; }
                fast_forward();
                to_event = dots_to_event();
                if (frame * kFrameDots + frame_dot >= target) going = false;
            }
        }
        if (pend != 0) settle(pend);
        pend = 0;
        // MMC2: the latches the frozen frame's fetches left, resolved after the vblank stop (nothing runs between the
        // two; rl/csrc/rlenv_core.cuh:161-176 does the same) by every lane that froze one, together
        if constexpr (BOARD == kMmc2) { if (froze) mmc2_resolve(); }
        return fault;
    }

    // End of a frame: presentation slot `slot` holds the last frozen frame (copied forward when no vblank froze one
    // during this frame, e.g. a faulted console).
    __device__ __forceinline__ void finish_slot() {
        const u32 fs = rw(R_FSLOT);
        if (fs == slot) return;
        const u64 a0 = static_cast<u64>(e) * 4 + fs, b0 = static_cast<u64>(e) * 4 + slot;
        copy16(S.snap_nt + b0 * kNtBytes, S.snap_nt + a0 * kNtBytes, kNtBytes);
        copy16(S.snap_oam + b0 * kOamBytes, S.snap_oam + a0 * kOamBytes, kOamBytes);
        if (S.snap_chr && !C.chr) {
            const bool shared = S.chr_ref && S.chr_ref[a0] != 0u;
            if (S.chr_ref) S.chr_ref[b0] = shared ? 1u : 0u;
            if (!shared) copy16(S.snap_chr + b0 * kChrRamBytes, S.snap_chr + a0 * kChrRamBytes, kChrRamBytes);
        }
        S.slot_bank[b0] = S.slot_bank[a0];
        ww(R_FSLOT, slot);
    }
};

// ------------------------------------------------------------------------------------------------ sprite-0 hit
// FCEUmm's sprite-0 hit from the frame log written so far (patch:1740-1789 frame_sprite0_hit): the replay of lines 0
// to sprite 0's last line with the check at each line's end. Exact, with closed forms where the log does not touch
// a line: lines above sprite 0 only step the PPU address (no memory access), and a line drawn without writes needs
// only the two background tiles under sprite 0. Lines with writes inside their drawn part take the exact tile loop.
// Out of line and by value, so the emulator's registers never have their address taken.

struct S0Ctx {
    const u32* bank;      // the writing log bank
    u32 count;
    const u8* nt;         // live nametable RAM of the env
    const u32* soam;      // OAM word 0 of the env's shared column (stride kEnvsPerWarp words)
    const u8* chr;        // CHR ROM (nullptr: chr_ram)
    const u8* chr_ram;    // the env's CHR-RAM
    u32 chr_size, chr_page_mask, arrangement;
};

struct S0State {
    u32 v, t, x, ctrl, mask, mirroring;
    u32 chr[8];
    u32 cursor;
    u32 sh0, sh1, at;          // tile shift registers after the last drawn tiles
    u32 lazy, lz_v, lz_ctrl;   // shift registers not yet materialised: fetches 32 / 33 of the line at lz_v
    u32 lz_chr[8], lz_mirroring;
    u32 blurp, f_lo0, f_hi0, f_attr0, f_x0;
    u32 sphitx, sphitdata, hit, hit_x;
    u32 latch[2], creg[4];     // MMC2: the latches and CHR registers of the replay
    u32 lz_chr33[8];           // MMC2: the pages fetch 33 of the lazy line went through (a fetch-32 flip moves them)
};

template <u32 BOARD>
__device__ __forceinline__ u32 s0_chr(const S0Ctx& c, const u32* chr_pages, u32 addr) {
    addr &= 0x1FFFu;
    if constexpr (board_paged(BOARD)) {
        const u32 off = ((chr_pages[addr >> 10] & c.chr_page_mask) << 10) | (addr & 0x3FFu);
        return c.chr ? __ldg(c.chr + off) : c.chr_ram[off & 0x1FFFu];
    } else {
        return c.chr ? __ldg(c.chr + (addr % c.chr_size)) : c.chr_ram[addr];
    }
}

// One tile fetch at PPU address v: lo | hi << 8 | attribute << 16.
template <u32 BOARD>
__device__ __forceinline__ u32 s0_fetch(const S0Ctx& c, u32 ctrl, const u32* chr_pages, u32 mirroring, u32 v) {
    auto ntrd = [&](u32 addr) -> u32 {
        if constexpr (board_paged(BOARD)) return c.nt[nt_off_map(mirroring, addr)];
        else return c.nt[nt_off_header(c.arrangement, addr)];
    };
    const u32 base = 0x2000u | (v & 0x0C00u);
    const u32 tile = ntrd(base | (v & 0x3FFu));
    const u32 zz = v & 0x1Fu;
    const u32 ab = ntrd(base | 0x3C0u | (zz >> 2) | ((v & 0x380u) >> 4));
    const u32 cc = (ab >> ((zz & 2u) + ((v & 0x40u) >> 4))) & 3u;
    const u32 vadr = (tile << 4) + (((ctrl & 0x10u) << 8) | ((v >> 12) & 7u));
    return s0_chr<BOARD>(c, chr_pages, vadr) | (s0_chr<BOARD>(c, chr_pages, vadr + 8u) << 8) | (cc << 16);
}

// MMC2 in the replay (patch:1385-1402): a half's four 1 KB pages from the register its latch picks; the hook on a
// fetched pattern address in $0FD0-$0FEF / $1FD0-$1FEF puts that half on its $FD or $FE bank.
// The low-plane pattern address of the tile fetch at PPU address v.
template <u32 BOARD>
__device__ __forceinline__ u32 s0_tile_addr(const S0Ctx& c, u32 ctrl, u32 mirroring, u32 v) {
    u32 tile;
    if constexpr (board_paged(BOARD)) tile = c.nt[nt_off_map(mirroring, 0x2000u | (v & 0x0FFFu))];
    else tile = c.nt[nt_off_header(c.arrangement, 0x2000u | (v & 0x0FFFu))];
    return (tile << 4) + (((ctrl & 0x10u) << 8) | ((v >> 12) & 7u));
}

__device__ __forceinline__ void s0_mmc2_select(S0State& s, u32 half) {
    const u32 bank = s.creg[(2 * half + (s.latch[half & 1u] & 1u)) & 3u];   // an index within the array always
    for (u32 i = 0; i < 4; ++i) s.chr[4 * half + i] = (bank * 4 + i) & 0xFFu;
}
__device__ __forceinline__ void s0_mmc2_hook(S0State& s, u32 addr) {
    const u32 high = (addr >> 8) & 0xFFu, low = addr & 0xF0u;
    if (high >= 0x20u || (high & 0x0Fu) != 0x0Fu || (low != 0xD0u && low != 0xE0u)) return;
    const u32 half = high >> 4;
    s.latch[half] = low == 0xE0u ? 1u : 0u;
    s0_mmc2_select(s, half);
}

template <u32 BOARD>
__device__ __forceinline__ void s0_apply(S0State& s, const u32* ev, u32 i, bool drawing) {
    const u32 w1 = ev[2 * i + 1];
    const u32 value = w1 & 0xFFu, aux = (w1 >> 8) & 0xFFu;
    const u32 inc = (s.ctrl & 4u) ? 32u : 1u;
    switch (ev[2 * i] >> 24) {
        case kEvCtrl: s.ctrl = value; s.t = (s.t & 0xF3FFu) | ((value & 3u) << 10); break;
        case kEvMask: s.mask = value; break;
        case kEvScroll:
            if (aux == 0) { s.t = (s.t & 0xFFE0u) | (value >> 3); s.x = value & 7u; }
            else s.t = (s.t & 0x8C1Fu) | ((value & 0xF8u) << 2) | ((value & 7u) << 12);
            break;
        case kEvAddr:
            if (aux == 0) s.t = (s.t & 0x00FFu) | ((value & 0x3Fu) << 8);
            else { s.t = (s.t & 0xFF00u) | value; s.v = s.t; }
            break;
        case kEvDataWrite: s.v = (s.v + (aux + 1u) * inc) & 0x7FFFu; break;
        case kEvDataRead:
            if (drawing && (s.mask & 0x18u)) s.v = v_inc_y(s.v);
            else s.v = (s.v + inc) & 0x7FFFu;
            break;
        case kEvPalette: s.v = (s.v + inc) & 0x7FFFu; break;
        case kEvChr: s.chr[aux & 7u] = value; break;
        case kEvMirror: s.mirroring = value; break;
        case kEvMmc2:
            if constexpr (BOARD == kMmc2) {
                if (aux < 4u) { s.creg[aux] = value; s0_mmc2_select(s, aux >> 1); }
                else if (aux == 6u || aux == 7u) { s.latch[aux - 6u] = value & 1u; s0_mmc2_select(s, aux - 6u); }
            }
            break;
        default: break;
    }
}

template <u32 BOARD>
__device__ void s0_materialize(const S0Ctx& c, S0State& s) {
    if (!s.lazy) return;
    const u32 f32 = s0_fetch<BOARD>(c, s.lz_ctrl, s.lz_chr, s.lz_mirroring, v_inc_x_n(s.lz_v, 32));
    const u32 f33 = s0_fetch<BOARD>(c, s.lz_ctrl, BOARD == kMmc2 ? s.lz_chr33 : s.lz_chr, s.lz_mirroring,
                                    v_inc_x_n(s.lz_v, 33));
    s.sh0 = ((f32 & 0xFFu) << 8) | (f33 & 0xFFu);
    s.sh1 = (((f32 >> 8) & 0xFFu) << 8) | ((f33 >> 8) & 0xFFu);
    s.at = ((f32 >> 16) & 3u) | (((f33 >> 16) & 3u) << 2);
    s.lazy = 0;
}

// The exact FCEUmm tile loop of one line with writes landing inside it: keeps each drawn pixel's "opaque
// background" bit, which is all the sprite-0 check reads.
template <u32 BOARD>
__device__ void s0_event_line(const S0Ctx& c, S0State& s, int kook, int l, bool pixels) {
    s0_materialize<BOARD>(c, s);
    const u32* ev = c.bank + kLogHdr;
    u32 opq[8];
    for (int i = 0; i < 8; ++i) opq[i] = 0;
    const int start = l * 341 - 16;
    int firsttile = 0, outpos = 0;
    bool tofix = true;
    auto tiles = [&](int last) {
        const int first = firsttile;
        if (!(s.mask & 0x18u)) { outpos += 8 * (last - first); firsttile = last; return; }
        for (int tile = first; tile < last; ++tile) {
            if (tile >= 2) {
                if (pixels && outpos < 256) {
                    const u32 lo = ((s.sh0 >> (8 - s.x)) & 0xFFu), hi = ((s.sh1 >> (8 - s.x)) & 0xFFu);
                    const u32 o = lo | hi;
                    for (int k = 0; k < 8; ++k) {
                        const int px = outpos + k;
                        const u32 bit = (o >> (7 - k)) & 1u;
                        opq[px >> 5] = (opq[px >> 5] & ~(1u << (px & 31))) | (bit << (px & 31));
                    }
                }
                outpos += 8;
            }
            const u32 f = s0_fetch<BOARD>(c, s.ctrl, s.chr, s.mirroring, s.v);   // both bytes before the hook
            if constexpr (BOARD == kMmc2) s0_mmc2_hook(s, s0_tile_addr<BOARD>(c, s.ctrl, s.mirroring, s.v));
            s.at = ((s.at >> 2) | (((f >> 16) & 3u) << 2)) & 0xFu;
            s.sh0 = ((s.sh0 << 8) | (f & 0xFFu)) & 0xFFFFu;
            s.sh1 = ((s.sh1 << 8) | ((f >> 8) & 0xFFu)) & 0xFFFFu;
            s.v = v_inc_x(s.v);
        }
        if (pixels) {
            if (first <= 2 && 2 < last && !(s.mask & 0x02u)) opq[0] &= ~0xFFu;
            if (!(s.mask & 0x08u)) {
                int ts = first - 2, tc = last - first;
                if (ts < 0) { tc += ts; ts = 0; }
                for (int px = ts * 8; px < (ts + tc) * 8 && px < 256; ++px) opq[px >> 5] &= ~(1u << (px & 31));
            }
        }
        firsttile = last;
    };
    auto check = [&](int pp) {
        if (s.sphitx == 0x100u) return;
        for (int xx = static_cast<int>(s.sphitx); xx < static_cast<int>(s.sphitx) + 8 && xx < pp - 16 && xx < 255; ++xx) {
            if ((s.sphitdata & (0x80u >> (xx - s.sphitx))) && ((opq[xx >> 5] >> (xx & 31)) & 1u)) {
                s.hit = 1; s.hit_x = static_cast<u32>(xx); s.sphitx = 0x100u; return;
            }
        }
    };
    auto update = [&](int pp) {
        int last = pp >> 3;
        if (pixels && s.sphitx != 0x100u && static_cast<int>(s.sphitx) < pp - 16 && !(static_cast<int>(s.sphitx) < (last - 2) * 8)) ++last;
        if (last > 34) last = 34;
        if (last <= firsttile) return;
        tiles(last);
        if (pp >= 268 && tofix) { if (s.mask & 0x18u) s.v = v_inc_y(s.v); tofix = false; }
        if (pixels) check(pp);
    };
    while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 272) {
        const u32 kind = ev[2 * s.cursor] >> 24;
        if (kind != kEvDataWrite && kind != kEvPalette)
            update(fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) + 3 * static_cast<int>((ev[2 * s.cursor] >> 17) & 0xFu) - start);
        s0_apply<BOARD>(s, ev, s.cursor++, true);
    }
    update(272);
    if (tofix) { if (s.mask & 0x18u) s.v = v_inc_y(s.v); tofix = false; }
    if (pixels) check(272);
}

// The hit found at pixel x of line l (sphitx: where the check started): the frame dot from which an instruction sees
// the flag, FCEUmm's RefreshLine drawing one tile more while the check is pending (patch:1758-1770).
__device__ __forceinline__ Hit0 s0_hit_at(int l, u32 x, u32 sphitx) {
    const int hx = static_cast<int>(x), spx = static_cast<int>(sphitx);
    int pp = hx + 17;
    for (;; ++pp) {
        int lastt = pp >> 3;
        if (spx < pp - 16 && !(spx < (lastt - 2) * 8)) ++lastt;
        if (lastt > 34) lastt = 34;
        if (hx < (lastt - 2) * 8) break;
    }
    return Hit0{nesle_dot(l * 341 - 16 + pp - 12), true};
}

template <u32 BOARD>
__device__ __noinline__ Hit0 sprite0_hit(const S0Ctx c) {
    const u32* h = c.bank;
    const u32* ev = h + kLogHdr;
    const int kook = (h[15] & kLogKook) ? 1 : 0;
    auto oamb = [&](u32 i) -> u32 { return reinterpret_cast<const u8*>(c.soam + (i >> 2) * kEnvsPerWarp)[i & 3u]; };
    const u32 oy = oamb(0), otile = oamb(1), oattr = oamb(2), ox = oamb(3);
    const int first = static_cast<int>(oy) + 1;
    if (first >= 240) return Hit0{0, false};
    S0State s;
    s.ctrl = h[1] & 0xFFu; s.mask = (h[1] >> 8) & 0xFFu; s.x = (h[1] >> 16) & 7u;
    s.v = h[2] & 0x7FFFu; s.t = (h[2] >> 16) & 0x7FFFu;
    for (int i = 0; i < 8; ++i) s.chr[i] = (h[3 + (i >> 2)] >> ((i & 3) * 8)) & 0xFFu;
    s.mirroring = h[5] & 0xFFu;
    s.cursor = 0;
    s.sh0 = s.sh1 = s.at = 0;
    s.lazy = 0; s.lz_v = 0; s.lz_ctrl = 0; s.lz_mirroring = 0;
    for (int i = 0; i < 8; ++i) s.lz_chr[i] = 0;
    s.blurp = 0; s.f_lo0 = s.f_hi0 = s.f_attr0 = s.f_x0 = 0;
    s.sphitx = 0x100u; s.sphitdata = 0; s.hit = 0; s.hit_x = 0;
    s.latch[0] = s.latch[1] = 0;   // MMC2 fields: unused by this replay (MMC2 has its own), defined all the same
    for (int i = 0; i < 4; ++i) s.creg[i] = 0;
    for (int i = 0; i < 8; ++i) s.lz_chr33[i] = 0;
    while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < -16) s0_apply<BOARD>(s, ev, s.cursor++, false);
    if (s.mask & 0x18u) s.v = s.t;
    const int last = first + 15 < 239 ? first + 15 : 239;
    int l = 0;
    // lines above sprite 0 with no write anywhere in them: only the PPU address moves, in closed form (the lines
    // 0..k-1 whose ends come at or before the next event; events before -16 are applied, so next + 16 >= 0)
    {
        const int k = s.cursor < c.count
                          ? min(first - 1, max(0, fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) + 16) / 341)
                          : first - 1;
        if (k > 0 && (s.mask & 0x18u)) {
            const u32 th = s.t & 0x041Fu;
            s.lazy = 1; s.lz_ctrl = s.ctrl; s.lz_mirroring = s.mirroring;
            for (int i = 0; i < 8; ++i) s.lz_chr[i] = s.chr[i];
            s.lz_v = v_after_lines(s.v, static_cast<u32>(k - 1), th, true);
            s.v = v_after_lines(s.v, static_cast<u32>(k), th, true);
        }
        l = k;
    }
    for (; l <= last; ++l) {
        const int start = l * 341 - 16;
        const bool pixels = l >= first;
        const u32 sphitx0 = s.sphitx;
        if (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 272) {
            s0_event_line<BOARD>(c, s, kook, l, pixels);
        } else if (s.mask & 0x18u) {
            const u32 v0 = s.v;
            if (pixels && s.sphitx != 0x100u && (s.mask & 0x08u)) {
                // the (at most) two tiles under pixels sphitx..sphitx+7
                const u32 sx = s.sphitx;
                const u32 q = sx + s.x, j0 = q >> 3, r = q & 7u;
                const u32 fa = s0_fetch<BOARD>(c, s.ctrl, s.chr, s.mirroring, v_inc_x_n(v0, j0));
                const u32 fb = r ? s0_fetch<BOARD>(c, s.ctrl, s.chr, s.mirroring, v_inc_x_n(v0, j0 + 1)) : 0u;
                const u32 o16 = (((fa | (fa >> 8)) & 0xFFu) << 8) | ((fb | (fb >> 8)) & 0xFFu);
                u32 win = (o16 >> (8 - r)) & 0xFFu;               // bit 7 - k: pixel sx + k opaque
                if (sx < 8 && !(s.mask & 0x02u)) win &= (1u << sx) - 1u;     // left 8 pixels hidden
                if (sx + 8 > 255) win &= (0xFF00u >> (255 - sx)) & 0xFFu;
                const u32 hits = win & s.sphitdata;
                if (hits) { s.hit = 1; s.hit_x = sx + (__clz(hits) - 24); s.sphitx = 0x100u; }
            }
            s.lazy = 1; s.lz_v = v0; s.lz_ctrl = s.ctrl; s.lz_mirroring = s.mirroring;
            for (int i = 0; i < 8; ++i) s.lz_chr[i] = s.chr[i];
            s.v = v_inc_y(v_inc_x_n(v0, 34));
        }
        if (s.hit) return s0_hit_at(l, s.hit_x, sphitx0);
        // end of line: sprite fetch for line l + 1 (only sprite 0 matters), Fixit2, RefreshSprites
        s.sphitx = 0x100u;
        if ((s.mask & 0x18u) && l >= first - 1) {
            const u32 hgt = (s.ctrl & 0x20u) ? 16u : 8u;
            const u32 vofs = ((s.ctrl & 0x08u) && !(s.ctrl & 0x20u)) ? 0x1000u : 0u;
            const u32 tt = static_cast<u32>(l - static_cast<int>(oy));
            // blurp: sprite 0 is in range of line l + 1 (the count of other fetched sprites never changes the check)
            s.blurp = 0;
            if (tt < hgt) {
                s.blurp = 1;
                u32 vadr = hgt == 16u ? ((otile & 1u) << 12) + ((otile & 0xFEu) << 4) : (otile << 4) + vofs;
                if (oattr & 0x80u) { vadr += 7u; vadr -= tt; vadr += (s.ctrl & 0x20u) >> 1; vadr -= tt & 8u; }
                else { vadr += tt; vadr += tt & 8u; }
                vadr &= 0x1FFFu;
                s.f_lo0 = s0_chr<BOARD>(c, s.chr, vadr);
                s.f_hi0 = s0_chr<BOARD>(c, s.chr, vadr + 8u);
                s.f_attr0 = oattr; s.f_x0 = ox;
            }
        }
        while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 278) s0_apply<BOARD>(s, ev, s.cursor++, true);
        if (s.mask & 0x18u) s.v = (s.v & 0xFBE0u) | (s.t & 0x041Fu);
        while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 341) s0_apply<BOARD>(s, ev, s.cursor++, true);
        if ((s.mask & 0x10u) && s.blurp && !s.hit) {
            const u32 j = s.f_lo0 | s.f_hi0;
            if (j) { s.sphitx = s.f_x0; s.sphitdata = (s.f_attr0 & 0x40u) ? (__brev(j) >> 24) : j; }
        }
    }
    return Hit0{nesle_dot(last * 341 + 256), false};
}

// ------------------------------------------------------------------------------------------------ MMC2 latches
// MMC2's latches move with every pattern fetch the frame makes, so its sprite-0 replay and the vblank resolve
// (patch:1791-1815 frame_resolve_mmc2) follow the frame's fetch order. An event-free line's 34 background fetches all
// use one pattern table, so they can only move that half's latch, and only by a $FD or $FE tile number: the latch a
// fetch sees is the last such tile before it, else the one the line started with. The positions of those tiles are
// worked out once per run of lines with the same first fetch address, table and page map (the nametable does not
// change during the replay).

struct Mmc2Row { u32 key; u64 flips, fe; };   // bit k: fetch k reads a $FD / $FE tile; fe: which of them are $FE

template <u32 BOARD>
__device__ __forceinline__ void mmc2_row(const S0Ctx& c, const S0State& s, Mmc2Row& r) {
    const u32 key = 0x80000000u | (s.v & 0x0FFFu) | ((s.ctrl & 0x10u) << 8) | ((s.mirroring & 0xFFu) << 13);
    if (key == r.key) return;
    r.key = key;
    r.flips = r.fe = 0;
    for (u32 k = 0; k < 34; ++k) {
        const u32 vv = v_inc_x_n(s.v, k);
        const u32 tile = c.nt[nt_off_map(s.mirroring, 0x2000u | (vv & 0x0FFFu))];
        if (tile == 0xFDu || tile == 0xFEu) r.flips |= 1ull << k;
        if (tile == 0xFEu) r.fe |= 1ull << k;
    }
}

// The background half's latch that fetch k of the row sees (lin: the latch the line started with).
__device__ __forceinline__ u32 mmc2_latch_before(const Mmc2Row& r, u32 k, u32 lin) {
    const u64 m = r.flips & ((1ull << k) - 1ull);
    return m ? static_cast<u32>((r.fe >> (63 - __clzll(static_cast<long long>(m)))) & 1ull) : lin;
}

// An event-free line drawn with rendering on: its latch moves and the lazy shift-register record (fetch 32 through
// the pages before fetch 32's own flip, fetch 33 through those before its own), then the address steps.
template <u32 BOARD>
__device__ __forceinline__ void mmc2_plain_line(const S0Ctx& c, S0State& s, Mmc2Row& row, bool keep_lazy) {
    mmc2_row<BOARD>(c, s, row);
    const u32 bg = (s.ctrl >> 4) & 1u;
    const u32 lin = s.latch[bg];
    const u32 l32 = mmc2_latch_before(row, 32, lin);
    const u32 l33 = mmc2_latch_before(row, 33, lin);
    if (keep_lazy) {
        s.lazy = 1; s.lz_v = s.v; s.lz_ctrl = s.ctrl; s.lz_mirroring = s.mirroring;
        s.latch[bg] = l32; s0_mmc2_select(s, bg);
        for (int i = 0; i < 8; ++i) s.lz_chr[i] = s.chr[i];
        s.latch[bg] = l33; s0_mmc2_select(s, bg);
        for (int i = 0; i < 8; ++i) s.lz_chr33[i] = s.chr[i];
    }
    s.latch[bg] = mmc2_latch_before(row, 34, lin);
    s0_mmc2_select(s, bg);
    s.v = v_inc_y(v_inc_x_n(s.v, 34));
}

// Sprite-0 check on an event-free line drawn with rendering on (before mmc2_plain_line steps it): the (at most) two
// background tiles under pixels sphitx..sphitx+7, each through the pages its fetch saw.
template <u32 BOARD>
__device__ __forceinline__ void mmc2_plain_hit(const S0Ctx& c, S0State& s, Mmc2Row& row) {
    if (s.sphitx == 0x100u || !(s.mask & 0x08u)) return;
    mmc2_row<BOARD>(c, s, row);
    const u32 bg = (s.ctrl >> 4) & 1u, lin = s.latch[bg];
    const u32 sx = s.sphitx;
    const u32 q = sx + s.x, j0 = q >> 3, r = q & 7u;
    u32 pages[8];
    auto fetch_at = [&](u32 k) {
        const u32 bank = s.creg[(2 * bg + mmc2_latch_before(row, k, lin)) & 3u];
        for (u32 i = 0; i < 8; ++i) pages[i] = s.chr[i];
        for (u32 i = 0; i < 4; ++i) pages[4 * bg + i] = (bank * 4 + i) & 0xFFu;
        return s0_fetch<BOARD>(c, s.ctrl, pages, s.mirroring, v_inc_x_n(s.v, k));
    };
    const u32 fa = fetch_at(j0);
    const u32 fb = r ? fetch_at(j0 + 1) : 0u;
    const u32 o16 = (((fa | (fa >> 8)) & 0xFFu) << 8) | ((fb | (fb >> 8)) & 0xFFu);
    u32 win = (o16 >> (8 - r)) & 0xFFu;                          // bit 7 - k: pixel sx + k opaque
    if (sx < 8 && !(s.mask & 0x02u)) win &= (1u << sx) - 1u;     // left 8 pixels hidden
    if (sx + 8 > 255) win &= (0xFF00u >> (255 - sx)) & 0xFFu;
    const u32 hits = win & s.sphitdata;
    if (hits) { s.hit = 1; s.hit_x = sx + (__clz(hits) - 24); s.sphitx = 0x100u; }
}

// FetchSpriteData at the end of line l with rendering on: every sprite in range (at most 8, OAM order) goes through
// the latch hook; sprite 0's pattern bytes are kept for the hit check. `vis`: the OAM entries to look at (mmc2_begin).
template <u32 BOARD>
__device__ __forceinline__ void mmc2_sprites(const S0Ctx& c, S0State& s, int l, u64 vis) {
    auto oamb = [&](u32 i) -> u32 { return reinterpret_cast<const u8*>(c.soam + (i >> 2) * kEnvsPerWarp)[i & 3u]; };
    const u32 hgt = (s.ctrl & 0x20u) ? 16u : 8u;
    const u32 vofs = ((s.ctrl & 0x08u) && !(s.ctrl & 0x20u)) ? 0x1000u : 0u;
    u32 n = 0;
    s.blurp = 0;
    for (u64 m = vis; m; m &= m - 1) {
        const u32 i = static_cast<u32>(__ffsll(static_cast<long long>(m)) - 1);
        const u32 t = static_cast<u32>(l - static_cast<int>(oamb(4 * i)));
        if (t >= hgt) continue;
        if (n >= 8) break;
        ++n;
        const u32 tile = oamb(4 * i + 1), attr = oamb(4 * i + 2);
        u32 vadr = hgt == 16u ? ((tile & 1u) << 12) + ((tile & 0xFEu) << 4) : (tile << 4) + vofs;
        if (attr & 0x80u) { vadr += 7u; vadr -= t; vadr += (s.ctrl & 0x20u) >> 1; vadr -= t & 8u; }
        else { vadr += t; vadr += t & 8u; }
        vadr &= 0x1FFFu;
        if (i == 0) {   // both bytes through the bank before the hook
            s.blurp = 1;
            s.f_lo0 = s0_chr<BOARD>(c, s.chr, vadr);
            s.f_hi0 = s0_chr<BOARD>(c, s.chr, vadr + 8u);
            s.f_attr0 = attr;
            s.f_x0 = oamb(3);
        }
        s0_mmc2_hook(s, vadr);
    }
}

template <u32 BOARD>
__device__ __forceinline__ void mmc2_begin(const S0Ctx& c, S0State& s, int kook, u64& vis) {
    const u32* h = c.bank;
    s.ctrl = h[1] & 0xFFu; s.mask = (h[1] >> 8) & 0xFFu; s.x = (h[1] >> 16) & 7u;
    s.v = h[2] & 0x7FFFu; s.t = (h[2] >> 16) & 0x7FFFu;
    for (int i = 0; i < 8; ++i) s.chr[i] = (h[3 + (i >> 2)] >> ((i & 3) * 8)) & 0xFFu;
    s.mirroring = h[5] & 0xFFu;
    s.latch[0] = (h[5] >> 8) & 1u; s.latch[1] = (h[5] >> 16) & 1u;
    for (int i = 0; i < 4; ++i) s.creg[i] = (h[6] >> (8 * i)) & 0xFFu;
    s.cursor = 0;
    s.sh0 = s.sh1 = s.at = 0;
    s.lazy = 0; s.lz_v = 0; s.lz_ctrl = 0; s.lz_mirroring = 0;
    for (int i = 0; i < 8; ++i) { s.lz_chr[i] = 0; s.lz_chr33[i] = 0; }
    s.blurp = 0; s.f_lo0 = s.f_hi0 = s.f_attr0 = s.f_x0 = 0;
    s.sphitx = 0x100u; s.sphitdata = 0; s.hit = 0; s.hit_x = 0;
    const u32* ev = h + kLogHdr;
    while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < -16) s0_apply<BOARD>(s, ev, s.cursor++, false);
    if (s.mask & 0x18u) s.v = s.t;
    // the OAM entries that can be in range of a line (y < 240); with at most 8 of them the 8-sprite limit never
    // binds, and only sprite 0 and the sprites whose fetch can reach a latch address (tile $FC-$FF covers both
    // sprite heights) need a look
    u64 all = 0, rel = 1;
    for (u32 i = 0; i < 64; ++i) {
        const u32 w = c.soam[i * kEnvsPerWarp];
        if ((w & 0xFFu) < 240u) {
            all |= 1ull << i;
            if (((w >> 8) & 0xFFu) >= 0xFCu) rel |= 1ull << i;
        }
    }
    vis = __popcll(all) <= 8 ? (all & rel) : all;
}

// End of line l after its pixels: sprite fetch (rendering on), Fixit2, RefreshSprites' sprite-0 data.
template <u32 BOARD>
__device__ __forceinline__ void mmc2_end_of_line(const S0Ctx& c, S0State& s, int kook, int l, u64 vis) {
    const u32* ev = c.bank + kLogHdr;
    const int start = l * 341 - 16;
    s.sphitx = 0x100u;
    if (s.mask & 0x18u) mmc2_sprites<BOARD>(c, s, l, vis);
    while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 278) s0_apply<BOARD>(s, ev, s.cursor++, true);
    if (s.mask & 0x18u) s.v = (s.v & 0xFBE0u) | (s.t & 0x041Fu);
    while (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 341) s0_apply<BOARD>(s, ev, s.cursor++, true);
    if ((s.mask & 0x10u) && s.blurp && !s.hit) {
        const u32 j = s.f_lo0 | s.f_hi0;
        if (j) { s.sphitx = s.f_x0; s.sphitdata = (s.f_attr0 & 0x40u) ? (__brev(j) >> 24) : j; }
    }
}

// MMC2's sprite-0 hit (patch:1740-1789 with the MMC2 fetch rules): an event-free line moves the latches and the
// address and, from sprite 0's first line on, checks the two tiles under sprite 0 through the pages their fetches
// saw; a line with a write inside its drawn part is replayed tile by tile.
template <u32 BOARD>
__device__ __noinline__ Hit0 sprite0_hit_mmc2(const S0Ctx c) {
    const int kook = (c.bank[15] & kLogKook) ? 1 : 0;
    const int first = static_cast<int>(reinterpret_cast<const u8*>(c.soam)[0]) + 1;
    if (first >= 240) return Hit0{0, false};
    const u32* ev = c.bank + kLogHdr;
    S0State s;
    u64 vis;
    mmc2_begin<BOARD>(c, s, kook, vis);
    Mmc2Row row;
    row.key = 0;
    const int last = first + 15 < 239 ? first + 15 : 239;
    for (int l = 0; l <= last; ++l) {
        const int start = l * 341 - 16;
        const u32 sphitx0 = s.sphitx;
        const bool event_line = s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 272;
        if (event_line) {
            s0_event_line<BOARD>(c, s, kook, l, l >= first);
        } else if (s.mask & 0x18u) {
            if (l >= first) mmc2_plain_hit<BOARD>(c, s, row);
            mmc2_plain_line<BOARD>(c, s, row, true);
        }
        if (s.hit) return s0_hit_at(l, s.hit_x, sphitx0);
        mmc2_end_of_line<BOARD>(c, s, kook, l, vis);
    }
    return Hit0{nesle_dot(last * 341 + 256), false};
}

// The latches the frame's fetches leave (latch 0 | latch 1 << 1), replayed over the whole picture and the events
// after it (patch:1791-1815; rl/csrc/nes_machine.cuh:107-130 runs the same replay after the vblank stop).
template <u32 BOARD>
__device__ __noinline__ u32 mmc2_latches(const S0Ctx c) {
    const int kook = (c.bank[15] & kLogKook) ? 1 : 0;
    const u32* ev = c.bank + kLogHdr;
    S0State s;
    u64 vis;
    mmc2_begin<BOARD>(c, s, kook, vis);
    Mmc2Row row;
    row.key = 0;
    for (int l = 0; l < 240; ++l) {
        const int start = l * 341 - 16;
        if (s.cursor < c.count && fceumm_time(ev[2 * s.cursor] & 0x1FFFFu, kook) < start + 272)
            s0_event_line<BOARD>(c, s, kook, l, false);
        else if (s.mask & 0x18u)
            mmc2_plain_line<BOARD>(c, s, row, false);
        mmc2_end_of_line<BOARD>(c, s, kook, l, vis);
    }
    while (s.cursor < c.count) s0_apply<BOARD>(s, ev, s.cursor++, false);
    return s.latch[0] | (s.latch[1] << 1);
}

template <u32 BOARD>
__device__ __forceinline__ Hit0 Emu<BOARD>::sprite0_eval() const {
    S0Ctx c;
    c.bank = writing_bank();
    c.count = log_n < kLogEv ? log_n : kLogEv;
    c.nt = nt();
    c.soam = &sh.oam[0][lane];
    c.chr = C.chr;
    c.chr_ram = C.chr ? nullptr : chr_ram();
    c.chr_size = C.chr_size;
    c.chr_page_mask = C.chr_page_mask;
    c.arrangement = C.arrangement;
    if constexpr (BOARD == kMmc2) return sprite0_hit_mmc2<BOARD>(c);
    else return sprite0_hit<BOARD>(c);
}

// MMC2 after the vblank stop: the latches the frozen frame's own fetches left go back to the board (patch:1791-1815
// frame_resolve_mmc2; rl/csrc/nes_machine.cuh:107-130 resolve_mmc2_frozen reads the frozen log the same way).
template <u32 BOARD>
__device__ __forceinline__ void Emu<BOARD>::mmc2_resolve() {
    S0Ctx c;
    c.bank = log_bank(log_ctl & kLcBank);
    c.count = min(c.bank[0] & ~kLogOverflow, kLogEv);
    c.nt = nt();
    c.soam = &sh.oam[0][lane];
    c.chr = C.chr;
    c.chr_ram = nullptr;
    c.chr_size = C.chr_size;
    c.chr_page_mask = C.chr_page_mask;
    c.arrangement = C.arrangement;
    const u32 latches = mmc2_latches<BOARD>(c);
    for (u32 half = 0; half < 2; ++half) {
        if (mreg(6u + half) != ((latches >> half) & 1u)) {
            set_mreg(6u + half, (latches >> half) & 1u);
            mmc2_chr4(half);
        }
    }
}

}  // namespace gr
