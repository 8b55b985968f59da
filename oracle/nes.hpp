// TEST INFRASTRUCTURE ONLY - the CPU oracle. Nothing in the product may include, link or call this file; only
// tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it (through liboracle_rlenv.so).
//
// One NES console as a plain struct (array-of-structures, one env at a time), restating the emulator the reference
// environment runs (NeSLE batch code + third_party/nesle-extensions.patch, driven by rl/csrc/nes_machine.cuh).
//
// Parity status. The patch pins, and this file follows line by line in behaviour:
//   * the frame log and the FCEUmm line replay (patch:894-1821, batch_frame.cuh),
//   * the lazy PPU timing events, sprite-0 replay, short ("kook") frames, MMC3 clocks (patch:1822-2240),
//   * the bus hooks that log PPU writes and board writes (patch:570-780), the DMC (patch:400-569),
//   * the paged boards MMC1/MMC2/MMC3 (patch:2841-3367) and the frame loop step_until
//     (rl/csrc/nes_machine.cuh:67-103); MMC2's latches the frame's fetches leave are resolved at vblank
//     (patch:1791-1815 frame_resolve_mmc2; rl/csrc/nes_machine.cuh:107-130 runs the same replay after the stop).
// NeSLE's base tree is not vendored (github.com/hbofz/NeSLE @ 0b04d8b9, cloned by scripts/setup_nesle.sh:9-19), so
// the 6502 core, the $2002/$2004/$2007 read side, OAM DMA length, the controller port, the UxROM window and cold
// reset are restated here from public 6502/NES documentation: PARITY UNPINNED against NeSLE for those parts. The
// CUDA product implements the same definitions independently; tests hold the two bit-exact.
#pragma once
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace orc {

using u8 = std::uint8_t;
using u16 = std::uint16_t;
using u32 = std::uint32_t;
using u64 = std::uint64_t;

// ------------------------------------------------------------------------------------------------ constants

constexpr u32 kDots = 341, kLines = 262, kFrameDots = kDots * kLines;   // 89342
constexpr u32 kVblankDot = 241 * kDots + 1;                             // NMI (rl/csrc/nes_machine.cuh:29)
constexpr u32 kPreRenderDot = 261 * kDots + 1;                          // pre-render settle: log capture
constexpr u32 kVblankFlagDot = kVblankDot - 12;                         // FCEUmm flag time (patch:1964-1972)
constexpr u32 kStatusClearDot = kPreRenderDot - 12;
constexpr u32 kMmc3VisibleClock = 266, kMmc3PreRenderClock = 256;       // patch:1868-1869
constexpr int kFceummOffset = 11;                                       // patch:951
constexpr u32 kLogHeader = 16, kLogEvents = 256, kLogBank = kLogHeader + 2 * kLogEvents;
constexpr u32 kLogOverflow = 0x80000000u, kLogKook = 0x100u;
constexpr u8 kLogNextKook = 2, kLogShortFrame = 4;
enum : u8 { kEvCtrl = 1, kEvMask, kEvScroll, kEvAddr, kEvDataWrite, kEvDataRead, kEvPalette, kEvChr, kEvMirror,
            kEvMmc2 };
constexpr u32 kS0Evaluate = 0x80000000u, kS0Known = 0x40000000u, kS0Hit = 0x20000000u, kS0DotMask = 0x1FFFFu;
constexpr u64 kDmcIdle = ~0ull;
constexpr u8 kPageVertical = 0x0A, kPageHorizontal = 0x0C, kPageSingleLow = 0x00, kPageSingleHigh = 0x0F;

enum Board : u8 { kNrom = 0, kUxrom = 1, kMmc1 = 2, kMmc3 = 3, kCnrom = 4, kMmc2 = 5 };
inline bool board_paged(Board b) { return b == kMmc1 || b == kMmc3 || b == kCnrom || b == kMmc2; }

// ------------------------------------------------------------------------------------------------ cartridge

struct Cart {
    std::vector<u8> prg;      // padded to a power of two
    std::vector<u8> chr;      // empty: 8 KB CHR-RAM per console
    u32 real_prg = 0;
    Board board = kNrom;
    u8 arrangement = 0;       // 0 vertical, 1 horizontal, 2 four-screen (header)
    u32 bank_mask = 0;        // UxROM 16 KB bank register mask
    u32 fixed_base = 0;       // UxROM: offset of the fixed last 16 KB
    u32 prg_page_mask = 0, chr_page_mask = 0;   // paged boards: 8 KB PRG pages - 1, 1 KB CHR pages - 1
};

// iNES 1.0 header -> cartridge (rl/csrc/rlenv_build.hpp:36-84 does the same through nesle::parse_ines and
// describe_mapper; the supported boards are the ones the benchmark configs use).
inline Cart parse_ines(const u8* rom, std::size_t n) {
    if (n < 16 || rom[0] != 'N' || rom[1] != 'E' || rom[2] != 'S' || rom[3] != 0x1A)
        throw std::runtime_error("not an iNES image");
    const u32 prg = rom[4] * 16384u, chr = rom[5] * 8192u;
    const u8 f6 = rom[6], f7 = rom[7];
    const u32 mapper = (f6 >> 4) | (f7 & 0xF0);
    const std::size_t off = 16 + ((f6 & 4) ? 512 : 0);
    if (prg == 0 || off + prg + chr > n) throw std::runtime_error("truncated iNES image");
    Cart c;
    c.real_prg = prg;
    u32 padded = 1;
    while (padded < prg) padded <<= 1;
    c.prg.assign(padded, 0);
    std::memcpy(c.prg.data(), rom + off, prg);
    c.chr.assign(rom + off + prg, rom + off + prg + chr);
    c.arrangement = (f6 & 8) ? 2 : (f6 & 1) ? 0 : 1;
    switch (mapper) {
        case 0:
            if (prg != 16384 && prg != 32768) throw std::runtime_error("NROM needs 16 or 32 KB PRG");
            if (chr == 0) throw std::runtime_error("NROM needs CHR ROM");
            c.board = kNrom;
            break;
        case 2:
            if (prg < 32768 || (prg & (prg - 1))) throw std::runtime_error("UxROM PRG must be a power of two");
            c.board = kUxrom;
            c.bank_mask = prg / 16384 - 1;
            c.fixed_base = prg - 16384;
            break;
        case 3:   // CNROM (patch:4007-4030 describe_mapper: PRG 16 KB - 512 KB in a power-of-two count of 8 KB pages,
                  // of which pages 0-3 are mapped; CHR ROM only, at most 256 KB)
            if (prg < 16384 || prg > 512 * 1024 || (prg & (prg - 1)) || chr == 0 || (chr & (chr - 1)) ||
                chr > 256 * 1024)
                throw std::runtime_error("unsupported CNROM image size");
            c.board = kCnrom;
            c.prg_page_mask = prg / 8192 - 1;
            c.chr_page_mask = chr / 1024 - 1;
            break;
        case 9:   // MMC2 (patch:4007-4030 describe_mapper: 8 KB PRG pages, CHR ROM only, at most 256 KB)
            if (prg < 32768 || prg > 512 * 1024 || (prg & (prg - 1)) || chr == 0 || (chr & (chr - 1)) ||
                chr > 256 * 1024)
                throw std::runtime_error("unsupported MMC2 image size");
            c.board = kMmc2;
            c.prg_page_mask = prg / 8192 - 1;
            c.chr_page_mask = chr / 1024 - 1;
            break;
        case 1:
        case 4: {
            c.board = mapper == 1 ? kMmc1 : kMmc3;
            const u32 chr_bytes = chr == 0 ? 8192u : chr;
            if (prg < 32768 || prg > 512 * 1024 || (prg & (prg - 1)) || (chr_bytes & (chr_bytes - 1)) ||
                chr_bytes > 256 * 1024)
                throw std::runtime_error("unsupported MMC1/MMC3 image size");
            c.prg_page_mask = prg / 8192 - 1;
            c.chr_page_mask = chr_bytes / 1024 - 1;
            break;
        }
        default:
            throw std::runtime_error("unsupported mapper " + std::to_string(mapper) +
                                     " (supported: 0 NROM, 1 MMC1, 2 UxROM, 3 CNROM, 4 MMC3, 9 MMC2)");
    }
    return c;
}

// ------------------------------------------------------------------------------------------------ console

struct Dmc {
    u64 byte_end;
    u16 bytes_left;
    u8 control, length, rate, buffer_full;
};

struct Console {
    // CPU (rl/csrc/nes_machine.cuh:40-44 bind_arrays order)
    u16 pc;
    u8 a, x, y, sp, p;
    u64 cycles;
    u8 cpu_nmi, irq_line;
    u8 ram[2048];
    u8 prg_ram[8192];
    u8 ctl_shift, ctl_count, ctl_strobe;
    u32 dma_pending;
    u32 fault, fault_pending;
    // PPU
    u8 ctrl, mask, status, oam_addr, nmi_pending;
    u32 frame_dot;
    u64 frame;
    u16 v, t;
    u8 fx, w, open_bus, read_buffer, scroll_x, scroll_y;
    u8 nt[2048], pal[32], oam[256];
    u8 chr_ram[8192];
    u32 log[2 * kLogBank];
    u16 log_count;
    u8 log_bank;
    u32 sprite0_dot;
    u8 snap_oam[256], snap_nt[2048];
    // board
    u8 prg_bank;
    u32 prg_page[4], chr_page[8];
    u8 mirroring;
    u8 regs[16];
    // APU sample channel
    u64 dmc_event;
    Dmc dmc;
    // pad byte the controller port presents this frame (BatchBuffers::action_masks)
    u8 pad;
    // frame dot at which the running instruction started (PpuHotState::now, patch:2142-2146); not saved state
    u32 now;
};

// ------------------------------------------------------------------------------------------------ mappers

namespace board {
enum : u32 { kMmc1Control = 0, kMmc1Chr0 = 1, kMmc1Chr1 = 2, kMmc1Prg = 3, kMmc1Shift = 4, kMmc1Count = 5 };
enum : u32 { kMmc2Prg = 4, kMmc2Mirror = 5, kMmc2Latch0 = 6, kMmc2Latch1 = 7 };   // r0-r3: CHR FD/FE, FD/FE
enum : u32 { kMmc3Select = 8, kMmc3Mirror = 9, kMmc3PrgRam = 10, kMmc3Latch = 11, kMmc3Counter = 12,
             kMmc3Enabled = 13, kMmc3Reload = 14 };

inline void prg8(const Cart& c, Console& m, u32 slot, u32 bank) { m.prg_page[slot] = (bank & c.prg_page_mask) << 13; }
inline void chr1(const Cart& c, Console& m, u32 slot, u32 bank) { m.chr_page[slot] = (bank & c.chr_page_mask) << 10; }
inline void prg16(const Cart& c, Console& m, u32 s, u32 b) { prg8(c, m, 2 * s, 2 * b); prg8(c, m, 2 * s + 1, 2 * b + 1); }
inline void chr4(const Cart& c, Console& m, u32 s, u32 b) { for (u32 i = 0; i < 4; ++i) chr1(c, m, 4 * s + i, 4 * b + i); }
inline void set_mirror(const Cart& c, Console& m, u8 map) { if (c.arrangement != 2) m.mirroring = map; }
inline u8 header_map(const Cart& c) { return c.arrangement == 1 ? kPageHorizontal : kPageVertical; }

// Page tables and mirroring from the registers (patch:2962-3054, mapper.cuh paged::sync).
inline void sync(const Cart& c, Console& m) {
    const u8* r = m.regs;
    if (c.board == kCnrom) {   // PRG pages 0-3 (mirrored through the mask), CHR 8 KB bank r[0] (patch:2982-2990)
        for (u32 s = 0; s < 4; ++s) prg8(c, m, s, s);
        for (u32 s = 0; s < 8; ++s) chr1(c, m, s, r[0] * 8u + s);
    } else if (c.board == kMmc1) {
        const u32 ctl = r[kMmc1Control], offs = r[kMmc1Chr0] & 0x10u, prg = r[kMmc1Prg];
        if ((ctl & 0x0C) == 0x0C) { prg16(c, m, 0, prg + offs); prg16(c, m, 1, 0x0F + offs); }
        else if ((ctl & 0x0C) == 0x08) { prg16(c, m, 1, prg + offs); prg16(c, m, 0, offs); }
        else { prg16(c, m, 0, (prg & ~1u) + offs); prg16(c, m, 1, (prg & ~1u) + offs + 1); }
        if (ctl & 0x10) { chr4(c, m, 0, r[kMmc1Chr0]); chr4(c, m, 1, r[kMmc1Chr1]); }
        else { chr4(c, m, 0, r[kMmc1Chr0] & 0xFEu); chr4(c, m, 1, r[kMmc1Chr0] | 1u); }
        const u8 maps[4] = {kPageSingleLow, kPageSingleHigh, kPageVertical, kPageHorizontal};
        set_mirror(c, m, maps[ctl & 3]);
    } else if (c.board == kMmc3) {
        const u32 sel = r[kMmc3Select], r6 = r[6] & 0x7Fu;
        if (sel & 0x40) { prg8(c, m, 2, r6); prg8(c, m, 0, 0x7E); }
        else { prg8(c, m, 0, r6); prg8(c, m, 2, 0x7E); }
        prg8(c, m, 1, r[7] & 0x7Fu);
        prg8(c, m, 3, 0x7F);
        const u32 f = (sel & 0x80) ? 4 : 0;
        chr1(c, m, 0 ^ f, r[0] & 0xFEu); chr1(c, m, 1 ^ f, r[0] | 1u);
        chr1(c, m, 2 ^ f, r[1] & 0xFEu); chr1(c, m, 3 ^ f, r[1] | 1u);
        chr1(c, m, 4 ^ f, r[2]); chr1(c, m, 5 ^ f, r[3]); chr1(c, m, 6 ^ f, r[4]); chr1(c, m, 7 ^ f, r[5]);
        set_mirror(c, m, (r[kMmc3Mirror] & 1) ? kPageHorizontal : kPageVertical);
    } else if (c.board == kMmc2) {   // patch:3027-3035: the switchable 8 KB page, then the last three
        prg8(c, m, 0, r[kMmc2Prg]);
        prg8(c, m, 1, ~2u);
        prg8(c, m, 2, ~1u);
        prg8(c, m, 3, ~0u);
        chr4(c, m, 0, r[r[kMmc2Latch0] & 1u]);
        chr4(c, m, 1, r[2u + (r[kMmc2Latch1] & 1u)]);
        set_mirror(c, m, r[kMmc2Mirror] ? kPageVertical : kPageHorizontal);
    }
}

// Power-on registers (patch:3057-3085).
inline void power_on(const Cart& c, Console& m) {
    std::memset(m.regs, 0, sizeof m.regs);
    m.mirroring = header_map(c);
    if (c.board == kMmc1) m.regs[kMmc1Control] = 0x0C;
    if (c.board == kMmc2) m.regs[kMmc2Latch0] = m.regs[kMmc2Latch1] = 1;   // both halves on their $FE bank
    if (c.board == kMmc3) {
        m.regs[1] = 2; m.regs[2] = 4; m.regs[3] = 5; m.regs[4] = 6; m.regs[5] = 7; m.regs[7] = 1;
        m.regs[kMmc3Mirror] = c.arrangement == 1 ? 1 : 0;
    }
    sync(c, m);
}

// CPU write to $8000-$FFFF on a paged board (patch:3099-3160).
inline void write(const Cart& c, Console& m, u16 addr, u8 value) {
    u8* r = m.regs;
    if (c.board == kCnrom) {   // the bank latch; an iNES 1.0 image declares no bus conflicts (patch:3124-3127)
        r[0] = value;
        sync(c, m);
        return;
    }
    if (c.board == kMmc1) {
        if (value & 0x80) { r[kMmc1Control] |= 0x0C; r[kMmc1Shift] = 0; r[kMmc1Count] = 0; sync(c, m); return; }
        r[kMmc1Shift] = static_cast<u8>(r[kMmc1Shift] | ((value & 1u) << r[kMmc1Count]));
        if (++r[kMmc1Count] < 5) return;
        r[(addr >> 13) - 4] = r[kMmc1Shift];
        r[kMmc1Shift] = 0;
        r[kMmc1Count] = 0;
        sync(c, m);
        return;
    }
    if (c.board == kMmc2) {   // patch:3147-3156
        switch (addr & 0xF000) {
            case 0xA000: r[kMmc2Prg] = value & 0x0F; break;
            case 0xB000: r[0] = value & 0x1F; break;
            case 0xC000: r[1] = value & 0x1F; break;
            case 0xD000: r[2] = value & 0x1F; break;
            case 0xE000: r[3] = value & 0x1F; break;
            case 0xF000: r[kMmc2Mirror] = (value & 1) ^ 1; break;
            default: return;   // $8000-$9FFF: no register
        }
        sync(c, m);
        return;
    }
    switch (addr & 0xE001) {
        case 0x8000: r[kMmc3Select] = value; break;
        case 0x8001: r[r[kMmc3Select] & 7] = value; break;
        case 0xA000: r[kMmc3Mirror] = value; break;
        case 0xA001: r[kMmc3PrgRam] = value; return;
        case 0xC000: r[kMmc3Latch] = value; return;
        case 0xC001: r[kMmc3Reload] = 1; return;
        case 0xE000: r[kMmc3Enabled] = 0; m.irq_line = 0; return;
        default: r[kMmc3Enabled] = 1; return;
    }
    sync(c, m);
}

// MMC2 latch hook: a PPU address in $0FD0-$0FEF / $1FD0-$1FEF puts that half on its $FD or $FE bank (FCEUmm's
// PPU_hook ranges, patch:3195-3222 mmc2_ppu_address). Returns the latch it changed + 1, or 0.
inline u32 mmc2_address(const Cart& c, Console& m, u32 addr) {
    const u32 high = (addr >> 8) & 0x3Fu, low = addr & 0xF0u;
    if (high >= 0x20u || (high & 0x0Fu) != 0x0Fu || (low != 0xD0u && low != 0xE0u)) return 0;
    const u32 half = high < 0x10u ? 0u : 1u;
    const u8 latch = low == 0xE0u ? 1 : 0;
    u8* r = m.regs;
    const u8 before = r[kMmc2Latch0 + half];
    r[kMmc2Latch0 + half] = latch;
    chr4(c, m, half, r[2u * half + latch]);
    return before != latch ? half + 1u : 0u;
}

// MMC3 counter clock, revision B (patch:3162-3174).
inline void mmc3_clock(Console& m) {
    u8* r = m.regs;
    if (r[kMmc3Counter] == 0 || r[kMmc3Reload]) { r[kMmc3Counter] = r[kMmc3Latch]; r[kMmc3Reload] = 0; }
    else --r[kMmc3Counter];
    if (r[kMmc3Counter] == 0 && r[kMmc3Enabled]) m.irq_line = 1;
}
}  // namespace board

inline u8 read_prg(const Cart& c, const Console& m, u16 addr) {
    switch (c.board) {
        case kNrom: return c.prg[(addr - 0x8000u) & (c.prg.size() - 1)];
        case kUxrom:
            return addr < 0xC000 ? c.prg[((m.prg_bank & c.bank_mask) << 14) | (addr & 0x3FFFu)]
                                 : c.prg[c.fixed_base + (addr & 0x3FFFu)];
        default: return c.prg[m.prg_page[(addr >> 13) & 3] + (addr & 0x1FFFu)];
    }
}

inline u8 read_chr(const Cart& c, const Console& m, u32 addr) {
    addr &= 0x1FFF;
    if (board_paged(c.board)) {
        const u32 off = m.chr_page[addr >> 10] + (addr & 0x3FF);
        return c.chr.empty() ? m.chr_ram[off & 0x1FFF] : c.chr[off];
    }
    return c.chr.empty() ? m.chr_ram[addr] : c.chr[addr % c.chr.size()];
}

inline void write_chr(const Cart& c, Console& m, u32 addr, u8 value) {
    if (!c.chr.empty()) return;
    addr &= 0x1FFF;
    if (board_paged(c.board)) addr = (m.chr_page[addr >> 10] + (addr & 0x3FF)) & 0x1FFF;
    m.chr_ram[addr] = value;
}

// CIRAM offset of $2000-$3EFF (four-screen folds to vertical: 2 KB of CIRAM, patch:3347-3355).
inline u32 nt_offset(const Cart& c, const Console& m, u32 addr) {
    const u32 index = (addr - 0x2000u) & 0x0FFFu;
    if (board_paged(c.board)) return (((m.mirroring >> (index >> 10)) & 1u) << 10) | (index & 0x3FFu);
    if (c.arrangement == 1) return (((index >> 11) & 1u) << 10) | (index & 0x3FFu);   // horizontal
    return index & 0x7FFu;                                                           // vertical / four-screen
}

inline bool prg_ram_enabled(const Cart& c, const Console& m) {
    return c.board != kMmc1 || (m.regs[board::kMmc1Prg] & 0x10) == 0;
}

// ------------------------------------------------------------------------------------------------ DMC (patch:430-565)

inline u32 dmc_period(u8 rate) {
    static const u16 t[16] = {428, 380, 340, 320, 286, 254, 226, 214, 190, 160, 142, 128, 106, 84, 72, 54};
    return t[rate & 15];
}

inline void dmc_reset(Console& m, u64 now) {
    m.dmc = Dmc{};
    m.dmc.byte_end = now + 1 + 7ull * dmc_period(0);
    m.dmc_event = kDmcIdle;
}

inline u32 dmc_service(Console& m, u64 now, bool steal) {
    Dmc& d = m.dmc;
    const u64 byte_cycles = 8ull * dmc_period(d.rate);
    auto skip = [&] { if (d.byte_end <= now) d.byte_end += ((now - d.byte_end) / byte_cycles + 1) * byte_cycles; };
    u32 stolen = 0;
    if (!d.buffer_full) skip();
    for (;;) {
        if (d.buffer_full) {
            if (d.byte_end > now) break;
            d.buffer_full = 0;
            d.byte_end += byte_cycles;
            if (d.bytes_left == 0) { skip(); break; }
        }
        if (d.bytes_left == 0) break;
        d.buffer_full = 1;
        if (--d.bytes_left == 0 && (d.control & 0x40)) d.bytes_left = static_cast<u16>(d.length * 16u + 1u);
        if (steal) { stolen += 4; now += 4; }
    }
    const u8 rate = d.control & 0x0F;
    if (rate != d.rate) {
        const u64 oldp = dmc_period(d.rate);
        const u64 later = (d.byte_end - now - 1) / oldp;
        d.byte_end = d.byte_end - later * oldp + later * dmc_period(rate);
        d.rate = rate;
    }
    m.dmc_event = d.buffer_full ? d.byte_end : kDmcIdle;
    return stolen;
}

inline void dmc_write(Console& m, u16 addr, u8 value) {
    Dmc& d = m.dmc;
    if (addr == 0x4010) d.control = value;
    else if (addr == 0x4013) d.length = value;
    else if (!(value & 0x10)) d.bytes_left = 0;
    else if (d.bytes_left == 0) d.bytes_left = static_cast<u16>(d.length * 16u + 1u);
    m.dmc_event = 0;
}

// ------------------------------------------------------------------------------------------------ frame log

inline int fceumm_time(u32 dot, int kook) {
    const int d = static_cast<int>(dot);
    return dot >= kPreRenderDot ? d - static_cast<int>(kFrameDots) + kFceummOffset + kook : d + kFceummOffset;
}
inline u32 nesle_dot(int fceumm) { return static_cast<u32>(fceumm - kFceummOffset); }

inline u32* log_bank_ptr(Console& m, u32 bank) { return m.log + bank * kLogBank; }
inline const u32* log_bank_ptr(const Console& m, u32 bank) { return m.log + bank * kLogBank; }

// Header of the state a frame starts from (patch:1047-1077).
inline void fill_header(const Cart& c, const Console& m, u8 ctrl, u8 mask, u32* h) {
    h[0] = 0;
    h[1] = ctrl | (u32(mask) << 8) | (u32(m.fx) << 16);
    h[2] = u32(m.v) | (u32(m.t) << 16);
    h[3] = h[4] = h[5] = h[6] = h[15] = 0;
    if (board_paged(c.board)) {
        for (u32 i = 0; i < 8; ++i) h[3 + (i >> 2)] |= ((m.chr_page[i] >> 10) & 0xFFu) << ((i & 3) * 8);
        h[5] = m.mirroring;
        if (c.board == kMmc2) {   // patch:1034-1040: latches in h[5], the four CHR registers in h[6]
            h[5] |= (u32(m.regs[board::kMmc2Latch0] & 1u) << 8) | (u32(m.regs[board::kMmc2Latch1] & 1u) << 16);
            h[6] = m.regs[0] | (u32(m.regs[1]) << 8) | (u32(m.regs[2]) << 16) | (u32(m.regs[3]) << 24);
        }
    }
    for (u32 i = 0; i < 8; ++i)
        h[7 + i] = m.pal[4 * i] | (u32(m.pal[4 * i + 1]) << 8) | (u32(m.pal[4 * i + 2]) << 16) |
                   (u32(m.pal[4 * i + 3]) << 24);
}

inline u8 log_capture(const Cart& c, Console& m) {
    u32* h = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    fill_header(c, m, m.ctrl, m.mask, h);
    const bool kook = (m.log_bank & kLogNextKook) != 0;
    if (kook) h[15] = kLogKook;
    return static_cast<u8>(((m.log_bank ^ kLogNextKook) & ~kLogShortFrame) | (kook ? kLogShortFrame : 0));
}

// FCEUmm's emphasis tint after a frame (patch:1087-1118).
inline u32 log_emphasis(const u32* h, u32 previous) {
    const u32* ev = h + kLogHeader;
    const u32 count = h[0] & ~kLogOverflow;
    u32 mask = (h[1] >> 8) & 0xFF;
    bool any = (mask & 0xE0) != 0;
    for (u32 i = 0; i < count && !any; ++i) any = (ev[2 * i] >> 24) == kEvMask && (ev[2 * i + 1] & 0xE0) != 0;
    if (!any) return previous;
    const int kook = (h[15] & kLogKook) ? 1 : 0;
    u32 i = 0;
    for (; i < count && fceumm_time(ev[2 * i] & 0x1FFFF, kook) < 0; ++i)
        if ((ev[2 * i] >> 24) == kEvMask) mask = ev[2 * i + 1] & 0xFF;
    u32 deemp = mask >> 5;
    u32 lines[8] = {};
    for (int l = 0; l < 240; ++l) {
        for (; i < count && fceumm_time(ev[2 * i] & 0x1FFFF, kook) < l * 341; ++i) {
            const u32 value = ev[2 * i + 1] & 0xFF;
            if ((ev[2 * i] >> 24) == kEvMask && (value & 0xE0)) deemp = value >> 5;
        }
        ++lines[deemp];
    }
    u32 most = 0, best = 0;
    for (u32 e = 1; e < 7; ++e) if (lines[e] > most) { most = lines[e]; best = e; }
    return best ? best : previous;
}

inline u8 log_freeze(Console& m, u16 log_n) {
    u32* h = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    const u32* shown = log_bank_ptr(m, m.log_bank & 1u);
    h[0] = (h[0] & kLogOverflow) | log_n;
    h[15] = (h[15] & ~7u) | log_emphasis(h, shown[15] & 7u);
    return static_cast<u8>(m.log_bank ^ 1u);
}

inline void log_reset(const Cart& c, Console& m) {
    fill_header(c, m, m.ctrl, m.mask, log_bank_ptr(m, 0));
    fill_header(c, m, m.ctrl, m.mask, log_bank_ptr(m, 1));
    m.log_count = 0;
    m.log_bank = 0;
    std::memcpy(m.snap_nt, m.nt, 2048);
    std::memcpy(m.snap_oam, m.oam, 256);
}

inline bool log_active(const Console& m) { return m.now < kVblankDot || m.now >= kPreRenderDot; }

inline void log_event(Console& m, u8 kind, u32 value, u32 aux = 0) {
    if (!log_active(m)) return;
    u32* bank = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    if (kind == kEvDataWrite && (m.mask & 0x18) == 0 && m.log_count != 0 && m.log_count <= kLogEvents) {
        u32* last = bank + kLogHeader + 2 * (m.log_count - 1u);
        if ((last[0] >> 24) == kEvDataWrite && (last[1] >> 8) < 0xFF) { last[1] += 0x100; return; }
    }
    if (m.log_count >= kLogEvents) { bank[0] |= kLogOverflow; return; }
    u32* e = bank + kLogHeader + 2 * m.log_count;
    e[0] = (m.now & 0x1FFFF) | (u32(kind) << 24);
    e[1] = (value & 0xFF) | ((aux & 0xFF) << 8);
    ++m.log_count;
}

inline void log_set_cycles(Console& m, u16 first, u32 cycles) {
    u32* bank = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    const u32 c = (cycles > 15 ? 15 : cycles) << 17;
    for (u32 i = first; i < m.log_count && i < kLogEvents; ++i) bank[kLogHeader + 2 * i] |= c;
}

// ------------------------------------------------------------------------------------------------ replay renderer
// FCEUmm's RefreshLine / FetchSpriteData / RefreshSprites / CopySprites / Fixit1 / Fixit2 / CheckSpriteHit replayed
// from a frame log (patch:1246-1738). Restated from the patch's description and code behaviour.

struct Src {
    const Cart* c;
    const Console* m;
    const u32* header;
    const u8* nt;
    const u8* oam;
    const u32* ev;
    u32 count;
    int kook;
};

inline Src make_src(const Cart& c, const Console& m, const u32* header, u32 count, const u8* nt, const u8* oam) {
    return Src{&c, &m, header, nt, oam, header + kLogHeader, count < kLogEvents ? count : kLogEvents,
               (header[15] & kLogKook) ? 1 : 0};
}

struct Sprites { u8 n; u8 lo[8], hi[8], attr[8], x[8]; };

struct RState {
    u16 v, t;
    u8 x, ctrl, mask, mirroring;
    u8 chr[8];
    u8 creg[4], latch[2];   // MMC2
    u8 pal[32];
    u32 sh0, sh1;
    u8 at;
    Sprites fetched;
    u8 blurp;
    Sprites drawn;
    u8 spal[16];
    u8 spork, hit, sphitdata;
    int sphitx, hit_x;
    u32 cursor;
};

struct RLine { u8 px[256]; int firsttile, outpos; bool tofix; };

inline int ev_start(const Src& s, u32 i) { return fceumm_time(s.ev[2 * i] & 0x1FFFF, s.kook); }
inline int ev_end(const Src& s, u32 i) { return ev_start(s, i) + 3 * static_cast<int>((s.ev[2 * i] >> 17) & 0xF); }
inline u32 ev_kind(const Src& s, u32 i) { return s.ev[2 * i] >> 24; }

inline void r_load(RState& s, const u32* h) {
    s.ctrl = static_cast<u8>(h[1]);
    s.mask = static_cast<u8>(h[1] >> 8);
    s.x = static_cast<u8>((h[1] >> 16) & 7);
    s.v = static_cast<u16>(h[2] & 0x7FFF);
    s.t = static_cast<u16>((h[2] >> 16) & 0x7FFF);
    for (int i = 0; i < 8; ++i) s.chr[i] = static_cast<u8>(h[3 + (i >> 2)] >> ((i & 3) * 8));
    s.mirroring = static_cast<u8>(h[5]);
    s.latch[0] = static_cast<u8>((h[5] >> 8) & 1);
    s.latch[1] = static_cast<u8>((h[5] >> 16) & 1);
    for (int i = 0; i < 4; ++i) s.creg[i] = static_cast<u8>(h[6] >> (8 * i));
    for (int i = 0; i < 32; ++i) s.pal[i] = static_cast<u8>(h[7 + (i >> 2)] >> ((i & 3) * 8));
    s.sh0 = s.sh1 = 0;
    s.at = 0;
    s.fetched.n = 0;
    s.blurp = 0;
    s.drawn.n = 0;
    s.spork = 0;
    s.hit = 0;
    s.sphitdata = 0;
    s.sphitx = 0x100;
    s.hit_x = -1;
    s.cursor = 0;
}

inline u8 r_chr(const Src& src, const RState& s, u32 addr) {
    const Cart& c = *src.c;
    addr &= 0x1FFF;
    if (board_paged(c.board)) {
        const u32 off = ((u32(s.chr[addr >> 10]) & c.chr_page_mask) << 10) | (addr & 0x3FF);
        return c.chr.empty() ? src.m->chr_ram[off & 0x1FFF] : c.chr[off];
    }
    return c.chr.empty() ? src.m->chr_ram[addr] : c.chr[addr % c.chr.size()];
}

inline u8 r_nt(const Src& src, const RState& s, u32 addr) {
    const Cart& c = *src.c;
    const u32 index = (addr - 0x2000u) & 0x0FFF;
    u32 off;
    if (board_paged(c.board)) off = (((s.mirroring >> (index >> 10)) & 1u) << 10) | (index & 0x3FF);
    else if (c.arrangement == 1) off = (((index >> 11) & 1u) << 10) | (index & 0x3FF);
    else off = index & 0x7FF;
    return src.nt[off];
}

inline bool r_on(const RState& s) { return (s.mask & 0x18) != 0; }

// MMC2 in the replay (patch:1385-1402): a half's four 1 KB pages from the register its latch picks, and the latch
// hook on every pattern address the frame fetches.
inline void r_mmc2_select(RState& s, u32 half) {
    const u32 bank = s.creg[2 * half + s.latch[half]];
    for (u32 i = 0; i < 4; ++i) s.chr[4 * half + i] = static_cast<u8>(bank * 4 + i);
}
inline void r_mmc2_hook(const Src& src, RState& s, u32 addr) {
    if (src.c->board != kMmc2) return;
    const u32 high = (addr >> 8) & 0xFF, low = addr & 0xF0;
    if (high >= 0x20 || (high & 0x0F) != 0x0F || (low != 0xD0 && low != 0xE0)) return;
    const u32 half = high < 0x10 ? 0 : 1;
    s.latch[half] = low == 0xE0 ? 1 : 0;
    r_mmc2_select(s, half);
}

inline void r_vinc(RState& s) {
    u32 v = s.v;
    if ((v & 0x7000) == 0x7000) {
        v ^= 0x7000;
        if ((v & 0x3E0) == 0x3A0) v ^= 0xBA0;
        else if ((v & 0x3E0) == 0x3E0) v ^= 0x3E0;
        else v += 0x20;
    } else {
        v += 0x1000;
    }
    s.v = static_cast<u16>(v & 0x7FFF);
}

inline void r_apply(const Src& src, RState& s, u32 i, bool drawing) {
    const u32 w1 = src.ev[2 * i + 1];
    const u32 value = w1 & 0xFF, aux = (w1 >> 8) & 0xFF;
    const u32 inc = (s.ctrl & 4) ? 32 : 1;
    switch (ev_kind(src, i)) {
        case kEvCtrl: s.ctrl = static_cast<u8>(value); s.t = static_cast<u16>((s.t & 0xF3FF) | ((value & 3) << 10)); break;
        case kEvMask: s.mask = static_cast<u8>(value); break;
        case kEvScroll:
            if (aux == 0) { s.t = static_cast<u16>((s.t & 0xFFE0) | (value >> 3)); s.x = static_cast<u8>(value & 7); }
            else s.t = static_cast<u16>((s.t & 0x8C1F) | ((value & 0xF8) << 2) | ((value & 7) << 12));
            break;
        case kEvAddr:
            if (aux == 0) s.t = static_cast<u16>((s.t & 0x00FF) | ((value & 0x3F) << 8));
            else { s.t = static_cast<u16>((s.t & 0xFF00) | value); s.v = s.t; }
            break;
        case kEvDataWrite: s.v = static_cast<u16>((s.v + (aux + 1) * inc) & 0x7FFF); break;
        case kEvDataRead:
            if (drawing && r_on(s)) r_vinc(s);
            else s.v = static_cast<u16>((s.v + inc) & 0x7FFF);
            break;
        case kEvPalette: s.pal[aux & 31] = static_cast<u8>(value); s.v = static_cast<u16>((s.v + inc) & 0x7FFF); break;
        case kEvChr: s.chr[aux & 7] = static_cast<u8>(value); break;
        case kEvMirror: s.mirroring = static_cast<u8>(value); break;
        case kEvMmc2:
            if (aux < 4) { s.creg[aux] = static_cast<u8>(value); r_mmc2_select(s, aux >> 1); }
            else if (aux == 6 || aux == 7) { s.latch[aux - 6] = static_cast<u8>(value & 1); r_mmc2_select(s, aux - 6); }
            break;
        default: break;
    }
}

inline void r_begin_frame(const Src& src, RState& s) {
    while (s.cursor < src.count && ev_start(src, s.cursor) < -16) r_apply(src, s, s.cursor++, false);
    if (r_on(s)) s.v = s.t;
}

// kLatchesOnly: the MMC2 resolve's replay, which needs the latches and nothing drawn (patch:1496-1526).
template <bool kLatchesOnly = false>
inline void r_tiles(const Src& src, RState& s, RLine& line, int last, bool pixels) {
    const int first = line.firsttile;
    const u8 backdrop = static_cast<u8>((s.pal[0] & 0x3F) | 0x40);
    if (!r_on(s)) {
        if (pixels)
            for (int p = line.outpos; p < line.outpos + 8 * (last - first) && p < 256; ++p) line.px[p] = backdrop;
        line.outpos += 8 * (last - first);
        line.firsttile = last;
        return;
    }
    int tile = first;
    if (!pixels && (kLatchesOnly || src.c->board != kMmc2)) {
        // no pixels: the address moves; only the last two tiles' fetches stay in the shift registers. MMC2's
        // latches see every pattern address, which needs only the tile number.
        for (; tile < last - 2; ++tile) {
            const u32 v = s.v;
            if (kLatchesOnly) {
                const u32 tidx = r_nt(src, s, 0x2000 | (v & 0x0FFF));
                r_mmc2_hook(src, s, (tidx << 4) + (((s.ctrl & 0x10u) << 8) | ((v >> 12) & 7)));
            }
            s.v = static_cast<u16>(((v & 0x1F) == 0x1F) ? (v ^ 0x41F) : (v + 1));
        }
    }
    for (; tile < last; ++tile) {
        if (tile >= 2) {
            if (pixels && line.outpos < 256) {
                const u32 lo = (s.sh0 >> (8 - s.x)) & 0xFF, hi = (s.sh1 >> (8 - s.x)) & 0xFF;
                for (int k = 0; k < 8; ++k) {
                    const u32 c = ((lo >> (7 - k)) & 1) | (((hi >> (7 - k)) & 1) << 1);
                    const u32 at = (k + s.x) < 8 ? (s.at & 3) : ((s.at >> 2) & 3);
                    line.px[line.outpos + k] = c == 0 ? backdrop : static_cast<u8>(s.pal[at * 4 + c] & 0x3F);
                }
            }
            line.outpos += 8;
        }
        const u32 v = s.v;
        const u32 base = 0x2000 | (v & 0x0C00);
        const u32 tidx = r_nt(src, s, base | (v & 0x3FF));
        const u32 zz = v & 0x1F;
        const u32 ab = r_nt(src, s, base | 0x3C0 | (zz >> 2) | ((v & 0x380) >> 4));
        const u32 cc = (ab >> ((zz & 2) + ((v & 0x40) >> 4))) & 3;
        const u32 vadr = (tidx << 4) + (((s.ctrl & 0x10u) << 8) | ((v >> 12) & 7));
        const u8 p0 = r_chr(src, s, vadr), p1 = r_chr(src, s, vadr + 8);   // both through the bank before the hook
        r_mmc2_hook(src, s, vadr);
        s.at = static_cast<u8>((s.at >> 2) | (cc << 2));
        s.sh0 = (s.sh0 << 8) | p0;
        s.sh1 = (s.sh1 << 8) | p1;
        s.v = static_cast<u16>(((v & 0x1F) == 0x1F) ? (v ^ 0x41F) : (v + 1));
    }
    if (pixels) {
        if (first <= 2 && 2 < last && (s.mask & 0x02) == 0) for (int p = 0; p < 8; ++p) line.px[p] = backdrop;
        if ((s.mask & 0x08) == 0) {
            int ts = first - 2, tc = last - first;
            if (ts < 0) { tc += ts; ts = 0; }
            for (int p = ts * 8; p < (ts + tc) * 8 && p < 256; ++p) line.px[p] = backdrop;
        }
    }
    line.firsttile = last;
}

inline void r_check_hit(RState& s, const RLine& line, int p) {
    if (s.sphitx == 0x100) return;
    for (int x = s.sphitx; x < s.sphitx + 8 && x < p - 16 && x < 255; ++x) {
        if ((s.sphitdata & (0x80u >> (x - s.sphitx))) && (line.px[x] & 0x40) == 0) {
            s.hit = 1;
            s.hit_x = x;
            s.sphitx = 0x100;
            return;
        }
    }
}

template <bool kLatchesOnly = false>
inline void r_update(const Src& src, RState& s, RLine& line, int p, bool pixels) {
    int last = p >> 3;
    if (pixels && s.sphitx != 0x100 && s.sphitx < p - 16 && !(s.sphitx < (last - 2) * 8)) ++last;
    if (last > 34) last = 34;
    if (last <= line.firsttile) return;
    r_tiles<kLatchesOnly>(src, s, line, last, pixels);
    if (p >= 268 && line.tofix) {
        if (r_on(s)) r_vinc(s);
        line.tofix = false;
    }
    if (pixels) r_check_hit(s, line, p);
}

template <bool kLatchesOnly = false>
inline void r_line(const Src& src, RState& s, RLine& line, int l, bool pixels) {
    const int start = l * 341 - 16;
    line.firsttile = 0;
    line.outpos = 0;
    line.tofix = true;
    if (pixels) std::memset(line.px, 0xFF, 256);
    while (s.cursor < src.count && ev_start(src, s.cursor) < start + 272) {
        const u32 kind = ev_kind(src, s.cursor);
        if (kind != kEvDataWrite && kind != kEvPalette)
            r_update<kLatchesOnly>(src, s, line, ev_end(src, s.cursor) - start, pixels);
        r_apply(src, s, s.cursor++, true);
    }
    r_update<kLatchesOnly>(src, s, line, 272, pixels);
    if (line.tofix) {
        if (r_on(s)) r_vinc(s);
        line.tofix = false;
    }
    if (pixels) r_check_hit(s, line, 272);
}

inline u32 r_compose(RState& s, RLine& line) {
    if ((s.mask & 0x10) && s.spork) {
        s.spork = 0;
        const Sprites& d = s.drawn;
        for (u32 xp = (s.mask & 0x04) ? 0 : 8; xp < 256; ++xp) {
            for (u32 n = 0; n < d.n; ++n) {
                const u32 k = xp - d.x[n];
                if (k >= 8) continue;
                const u32 bit = (d.attr[n] & 0x40) ? k : 7 - k;
                const u32 c = ((d.lo[n] >> bit) & 1) | (((d.hi[n] >> bit) & 1) << 1);
                if (c == 0) continue;
                if ((d.attr[n] & 0x20) == 0 || (line.px[xp] & 0x40)) line.px[xp] = s.spal[(d.attr[n] & 3) * 4 + c];
                break;
            }
        }
    }
    const u32 keep = (s.mask & 1) && r_on(s) ? 0x30 : 0x3F;
    for (int p = 0; p < 256; ++p) line.px[p] = static_cast<u8>(line.px[p] & keep);
    return s.mask >> 5;
}

inline void r_end_of_line(const Src& src, RState& s, int l, bool sprites) {
    const int start = l * 341 - 16;
    s.sphitx = 0x100;
    if (r_on(s) && (sprites || src.c->board == kMmc2)) {   // MMC2: every fetch moves the latches
        const u32 c = s.ctrl;
        const u32 h = (c & 0x20) ? 16 : 8;
        const u32 vofs = ((c & 0x08) && !(c & 0x20)) ? 0x1000 : 0;
        Sprites& f = s.fetched;
        f.n = 0;
        s.blurp = 0;
        for (u32 n = 0; n < 64; ++n) {
            const u8* spr = src.oam + 4 * n;
            const u32 t = static_cast<u32>(l - static_cast<int>(spr[0]));
            if (t >= h) continue;
            if (f.n >= 8) break;
            if (n == 0) s.blurp = 1;
            u32 vadr = h == 16 ? ((spr[1] & 1u) << 12) + ((spr[1] & 0xFEu) << 4) : (u32(spr[1]) << 4) + vofs;
            if (spr[2] & 0x80) { vadr += 7; vadr -= t; vadr += (c & 0x20) >> 1; vadr -= t & 8; }
            else { vadr += t; vadr += t & 8; }
            vadr &= 0x1FFF;
            f.lo[f.n] = r_chr(src, s, vadr);
            f.hi[f.n] = r_chr(src, s, vadr + 8);
            r_mmc2_hook(src, s, vadr);
            f.attr[f.n] = spr[2];
            f.x[f.n] = spr[3];
            ++f.n;
        }
    }
    while (s.cursor < src.count && ev_start(src, s.cursor) < start + 278) r_apply(src, s, s.cursor++, true);
    if (r_on(s)) s.v = static_cast<u16>((s.v & 0xFBE0) | (s.t & 0x041F));
    while (s.cursor < src.count && ev_start(src, s.cursor) < start + 341) r_apply(src, s, s.cursor++, true);
    if (s.mask & 0x10) {
        s.spork = 0;
        if (s.fetched.n) {
            s.drawn = s.fetched;
            for (int i = 0; i < 16; ++i) s.spal[i] = static_cast<u8>(s.pal[16 + i] & 0x3F);
            const u32 j = s.drawn.lo[0] | s.drawn.hi[0];
            if (s.blurp && !s.hit && j) {
                u32 data = j;
                if (s.drawn.attr[0] & 0x40) { data = 0; for (int k = 0; k < 8; ++k) data |= ((j >> k) & 1u) << (7 - k); }
                s.sphitx = s.drawn.x[0];
                s.sphitdata = static_cast<u8>(data);
            }
            s.spork = 1;
        }
    }
}

// Sprite-0 hit from the log written so far (patch:1740-1789).
struct Hit0 { u32 dot; bool hit; };

inline int sprite0_first_seen(int x, int sphitx) {
    for (int p = x + 17;; ++p) {
        int last = p >> 3;
        if (sphitx < p - 16 && !(sphitx < (last - 2) * 8)) ++last;
        if (last > 34) last = 34;
        if (x < (last - 2) * 8) return p;
    }
}

inline Hit0 sprite0_hit(const Cart& c, const Console& m) {
    const u32* h = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    const Src src = make_src(c, m, h, m.log_count, m.nt, m.oam);
    RState s;
    r_load(s, h);
    RLine line;
    const int first = static_cast<int>(src.oam[0]) + 1;
    if (first >= 240) return Hit0{0, false};
    r_begin_frame(src, s);
    const int last = first + 15 < 239 ? first + 15 : 239;
    for (int l = 0; l <= last; ++l) {
        const int sphitx = s.sphitx;
        r_line(src, s, line, l, l >= first);
        if (s.hit) return Hit0{nesle_dot(l * 341 - 16 + sprite0_first_seen(s.hit_x, sphitx) - 12), true};
        s.spork = 0;
        r_end_of_line(src, s, l, l >= first - 1);
    }
    return Hit0{nesle_dot(last * 341 + 256), false};
}

// MMC2 at vblank: the latches the frame's own tile and sprite fetches left (patch:1791-1815 frame_resolve_mmc2),
// replayed from the writing bank over the live nametable RAM and OAM (which hold what the frozen snapshots hold).
inline void resolve_mmc2(const Cart& c, Console& m) {
    const u32* h = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
    const Src src = make_src(c, m, h, m.log_count, m.nt, m.oam);
    RState s;
    r_load(s, h);
    RLine line;
    r_begin_frame(src, s);
    for (int l = 0; l < 240; ++l) {
        r_line<true>(src, s, line, l, false);
        r_end_of_line(src, s, l, true);
    }
    while (s.cursor < src.count) r_apply(src, s, s.cursor++, false);
    for (u32 half = 0; half < 2; ++half) {
        if (m.regs[board::kMmc2Latch0 + half] != s.latch[half]) {
            m.regs[board::kMmc2Latch0 + half] = s.latch[half];
            board::chr4(c, m, half, m.regs[2 * half + s.latch[half]]);
        }
    }
}

// The last frozen frame as colour numbers of the 240x224 crop + per-line emphasis (rl/csrc/nes_machine.cuh:133-155).
inline void render_obs(const Cart& c, const Console& m, u8* pix, u8* emph) {
    const u32* h = log_bank_ptr(m, m.log_bank & 1u);
    const Src src = make_src(c, m, h, h[0] & ~kLogOverflow, m.snap_nt, m.snap_oam);
    RState s;
    r_load(s, h);
    RLine line;
    r_begin_frame(src, s);
    for (int l = 0; l < 232; ++l) {
        r_line(src, s, line, l, true);
        const u32 e = r_compose(s, line);
        if (l >= 8) {
            const int y = l - 8;
            emph[y] = static_cast<u8>(e & 7);
            for (int x = 0; x < 240; ++x) pix[y * 240 + x] = line.px[8 + x] & 0x3F;
        }
        r_end_of_line(src, s, l, true);
    }
}

// ------------------------------------------------------------------------------------------------ PPU timing

// Dots to the next counter clock strictly after `cur` (patch:1881-1903).
inline u32 dots_to_mmc3_clock(u32 cur) {
    const u32 line = cur / kDots, dot = cur % kDots;
    if (line < 240) {
        if (dot < kMmc3VisibleClock) return kMmc3VisibleClock - dot;
        if (line + 1 < 240) return kDots - dot + kMmc3VisibleClock;
        return (261 - line) * kDots + kMmc3PreRenderClock - dot;
    }
    if (line < 261) return (261 - line) * kDots + kMmc3PreRenderClock - dot;
    if (dot < kMmc3PreRenderClock) return kMmc3PreRenderClock - dot;
    return kDots - dot + kMmc3VisibleClock;
}

inline void clock_mmc3(Console& m, u32 start, u32 end) {
    if ((m.mask & 0x18) == 0 || (m.ctrl & 0x38) == 0x18) return;
    for (u32 la = start / kDots; la <= end / kDots; ++la) {
        const u32 line = la % kLines;
        u32 cd;
        if (line < 240) cd = kMmc3VisibleClock;
        else if (line == 261) cd = kMmc3PreRenderClock;
        else continue;
        const u32 abs_dot = la * kDots + cd;
        if (abs_dot > start && abs_dot <= end) board::mmc3_clock(m);
    }
}

inline u32 dots_to_event(const Cart& c, const Console& m) {
    const u32 cur = m.frame_dot;
    const u32 skip = (m.log_bank & kLogShortFrame) ? 1 : 0;
    const u32 fd = kFrameDots - skip;
    auto dist = [&](u32 e) { return e > cur ? e - cur : fd - cur + e; };
    u32 next = fd - cur;
    auto take = [&](u32 d) { if (d < next) next = d; };
    take(dist(kVblankDot));
    take(dist(kPreRenderDot));
    take(dist(kVblankFlagDot));
    take(dist(kStatusClearDot));
    const u32 s0 = m.sprite0_dot & kS0DotMask;
    if (s0 != 0) take(dist(s0));
    if (c.board == kMmc3) {
        u32 clock = dots_to_mmc3_clock(cur);
        if (cur + clock >= kFrameDots) clock -= skip;
        take(clock);
    }
    return next;
}

// Settle the PPU by `dots` (patch:2114-2240 restated).
inline void ppu_settle(const Cart& c, Console& m, u32 dots) {
    const u32 start = m.frame_dot;
    const bool short_frame = (m.log_bank & kLogShortFrame) != 0;
    u32 end = start + dots;
    if (short_frame && end >= kFrameDots - 1) end += 1;
    const u32 frames = end / kFrameDots;
    for (u32 fo = 0; fo <= frames; ++fo) {
        auto crossed = [&](u32 ev) { const u32 a = fo * kFrameDots + ev; return a > start && a <= end; };
        const u32 sched = m.sprite0_dot;
        const u32 s0 = sched & kS0DotMask;
        if (s0 != 0 && crossed(s0)) {
            const bool known = (sched & kS0Known) && ((sched >> 20) & 0x1FF) == m.log_count;
            const Hit0 found = known ? Hit0{s0, (sched & kS0Hit) != 0} : sprite0_hit(c, m);
            const bool reached = fo * kFrameDots + found.dot <= end;
            if (found.hit && reached) m.status |= 0x40;
            m.sprite0_dot = found.dot != 0 && !reached
                                ? (found.dot | kS0Evaluate | kS0Known | (found.hit ? kS0Hit : 0u) | (u32(m.log_count) << 20))
                                : 0u;
        }
        if (crossed(kVblankFlagDot)) m.status |= 0x80;
        if (crossed(kVblankDot)) {
            if (m.ctrl & 0x80) m.nmi_pending = 1;
            if (c.board == kMmc2) resolve_mmc2(c, m);
            m.log_bank = log_freeze(m, m.log_count);
            std::memcpy(m.snap_oam, m.oam, 256);
            std::memcpy(m.snap_nt, m.nt, 2048);
        }
        if (crossed(kStatusClearDot)) { m.status &= 0x7F; m.status &= 0x1F; }
        if (crossed(kPreRenderDot)) {
            m.status &= 0x7F;
            m.status &= 0x1F;
            m.log_bank = log_capture(c, m);
            m.log_count = 0;
            const u32 y = m.oam[0];
            m.sprite0_dot = y < 239 ? (nesle_dot(static_cast<int>(y + 1) * 341 - 20) | kS0Evaluate) : 0u;
        }
    }
    if (c.board == kMmc3) clock_mmc3(m, start, end);
    m.frame_dot = end % kFrameDots;
    m.frame += frames;
    if (frames) m.log_bank &= static_cast<u8>(~kLogShortFrame);
}

// ------------------------------------------------------------------------------------------------ bus

inline u8 ppu_mem_read(const Cart& c, const Console& m, u32 addr) {
    addr &= 0x3FFF;
    if (addr < 0x2000) return read_chr(c, m, addr);
    if (addr < 0x3F00) return m.nt[nt_offset(c, m, addr >= 0x3000 ? addr - 0x1000 : addr)];
    u32 p = addr & 0x1F;
    if ((p & 0x13) == 0x10) p &= 0x0F;
    return m.pal[p];
}

inline u32 pal_index(u32 addr) { u32 p = addr & 0x1F; if ((p & 0x13) == 0x10) p &= 0x0F; return p; }

inline void ppu_mem_write(const Cart& c, Console& m, u32 addr, u8 value) {
    addr &= 0x3FFF;
    if (addr < 0x2000) { write_chr(c, m, addr, value); return; }
    if (addr < 0x3F00) { m.nt[nt_offset(c, m, addr >= 0x3000 ? addr - 0x1000 : addr)] = value; return; }
    m.pal[pal_index(addr)] = value;
}

inline void vram_inc(Console& m) { m.v = static_cast<u16>((m.v + ((m.ctrl & 4) ? 32 : 1)) & 0x7FFF); }

// The VRAM address the CPU puts on the PPU bus ($2006 / $2007): MMC2's latch hook, the change logged for the
// renderer while a frame is drawn (patch:615-636 bus_ppu_address).
inline void ppu_address(const Cart& c, Console& m, u32 addr) {
    if (c.board != kMmc2) return;
    if (const u32 changed = board::mmc2_address(c, m, addr)) {
        const u32 reg = board::kMmc2Latch0 + changed - 1;
        log_event(m, kEvMmc2, m.regs[reg], reg);
    }
}

inline u8 cpu_read(const Cart& c, Console& m, u16 addr) {
    if (addr < 0x2000) return m.ram[addr & 0x7FF];
    if (addr < 0x4000) {
        switch (addr & 7) {
            case 2: {
                const u8 value = static_cast<u8>((m.status & 0xE0) | (m.open_bus & 0x1F));
                m.status &= 0x7F;
                m.w = 0;
                return value;
            }
            case 4: return m.oam[m.oam_addr];
            case 7: {
                const u32 pa = m.v & 0x3FFF;
                u8 value;
                if (pa >= 0x3F00) {
                    value = ppu_mem_read(c, m, pa);
                    m.read_buffer = ppu_mem_read(c, m, pa - 0x1000);
                    ppu_address(c, m, pa);
                } else {
                    value = m.read_buffer;
                    ppu_address(c, m, pa);   // the buffer refills through the bank the address picks
                    m.read_buffer = ppu_mem_read(c, m, pa);
                }
                vram_inc(m);
                log_event(m, kEvDataRead, 0);
                ppu_address(c, m, m.v & 0x3FFF);
                m.open_bus = value;
                return value;
            }
            default: return 0;
        }
    }
    if (addr == 0x4015) return m.dmc.bytes_left ? 0x10 : 0x00;
    if (addr == 0x4016) {
        u32 bit;
        if (m.ctl_strobe) bit = m.pad & 1u;
        else if (m.ctl_count < 8) bit = (m.ctl_shift >> m.ctl_count++) & 1u;
        else bit = 1;
        return static_cast<u8>(0x40 | bit);
    }
    if (addr == 0x4017) return 0x40;
    if (addr < 0x6000) return static_cast<u8>(addr >> 8);
    if (addr < 0x8000) return prg_ram_enabled(c, m) ? m.prg_ram[addr - 0x6000] : static_cast<u8>(addr >> 8);
    return read_prg(c, m, addr);
}

inline void mapper_write(const Cart& c, Console& m, u16 addr, u8 value) {
    if (c.board == kUxrom) { m.prg_bank = static_cast<u8>(value & c.bank_mask); return; }
    if (!board_paged(c.board)) return;
    if (log_active(m)) {
        u32 before[8];
        for (int i = 0; i < 8; ++i) before[i] = m.chr_page[i];
        const u8 mir = m.mirroring;
        const u8 creg[4] = {m.regs[0], m.regs[1], m.regs[2], m.regs[3]};
        board::write(c, m, addr, value);
        for (u32 i = 0; i < 8; ++i) if (m.chr_page[i] != before[i]) log_event(m, kEvChr, m.chr_page[i] >> 10, i);
        if (m.mirroring != mir) log_event(m, kEvMirror, m.mirroring);
        if (c.board == kMmc2)   // the CHR registers a write changed (patch:661-665)
            for (u32 i = 0; i < 4; ++i) if (m.regs[i] != creg[i]) log_event(m, kEvMmc2, m.regs[i], i);
        return;
    }
    board::write(c, m, addr, value);
}

inline void cpu_write(const Cart& c, Console& m, u16 addr, u8 value) {
    if (addr < 0x2000) { m.ram[addr & 0x7FF] = value; return; }
    if (addr < 0x4000) {
        switch (addr & 7) {
            case 0:
                m.ctrl = value;
                m.t = static_cast<u16>((m.t & 0xF3FF) | ((value & 3) << 10));
                log_event(m, kEvCtrl, value);
                break;
            case 1: m.mask = value; log_event(m, kEvMask, value); break;
            case 3: m.oam_addr = value; break;
            case 4: m.oam[m.oam_addr++] = value; break;
            case 5:
                log_event(m, kEvScroll, value, m.w);
                if (m.w == 0) {
                    m.fx = value & 7;
                    m.t = static_cast<u16>((m.t & 0xFFE0) | (value >> 3));
                    m.scroll_x = value;
                    m.w = 1;
                } else {
                    m.t = static_cast<u16>((m.t & 0x8C1F) | ((value & 0xF8) << 2) | ((value & 7) << 12));
                    m.scroll_y = value;
                    m.w = 0;
                }
                break;
            case 6:
                log_event(m, kEvAddr, value, m.w);
                if (m.w == 0) { m.t = static_cast<u16>((m.t & 0x00FF) | ((value & 0x3F) << 8)); m.w = 1; }
                else { m.t = static_cast<u16>((m.t & 0x7F00) | value); m.v = m.t; m.w = 0; ppu_address(c, m, m.v); }
                break;
            case 7: {
                const u32 pa = m.v & 0x3FFF;
                ppu_mem_write(c, m, m.v, value);
                if (pa >= 0x3F00) log_event(m, kEvPalette, value, pal_index(pa));
                else log_event(m, kEvDataWrite, 0);
                vram_inc(m);
                ppu_address(c, m, m.v & 0x3FFF);
                break;
            }
            default: break;
        }
        m.open_bus = value;
        return;
    }
    if (addr == 0x4014) {
        const u16 base = static_cast<u16>(value << 8);
        for (u32 i = 0; i < 256; ++i) m.oam[(m.oam_addr + i) & 0xFF] = cpu_read(c, m, static_cast<u16>(base + i));
        m.dma_pending = 1;
        return;
    }
    if (addr == 0x4016) {
        m.ctl_strobe = value & 1;
        if (m.ctl_strobe) { m.ctl_shift = m.pad; m.ctl_count = 0; }
        return;
    }
    if (addr == 0x4010 || addr == 0x4013 || addr == 0x4015) { dmc_write(m, addr, value); return; }
    if (addr < 0x6000) return;
    if (addr < 0x8000) { if (prg_ram_enabled(c, m)) m.prg_ram[addr - 0x6000] = value; return; }
    mapper_write(c, m, addr, value);
}

// ------------------------------------------------------------------------------------------------ 6502

enum : u8 { FC = 1, FZ = 2, FI = 4, FD = 8, FB = 0x10, FU = 0x20, FV = 0x40, FN = 0x80 };

struct StepOut { u32 cycles; u8 opcode; u16 pc; bool illegal; };

struct Cpu {
    const Cart& c;
    Console& m;
    u8 rd(u16 a) { return cpu_read(c, m, a); }
    void wr(u16 a, u8 v) { cpu_write(c, m, a, v); }
    u16 rd16(u16 a) { return static_cast<u16>(rd(a) | (rd(static_cast<u16>(a + 1)) << 8)); }
    void push(u8 v) { m.ram[0x100 | m.sp] = v; --m.sp; }
    u8 pull() { ++m.sp; return m.ram[0x100 | m.sp]; }
    void nz(u8 v) { m.p = static_cast<u8>((m.p & ~(FZ | FN)) | (v == 0 ? FZ : 0) | (v & 0x80)); }
    void setf(u8 f, bool on) { m.p = static_cast<u8>(on ? (m.p | f) : (m.p & ~f)); }

    void interrupt(u16 vector) {
        push(static_cast<u8>(m.pc >> 8));
        push(static_cast<u8>(m.pc));
        push(static_cast<u8>((m.p & ~FB) | FU));
        m.p |= FI;
        m.pc = rd16(vector);
        m.cycles += 7;
    }

    void adc(u8 v) {
        const u32 s = u32(m.a) + v + (m.p & FC);
        setf(FV, (~(m.a ^ v) & (m.a ^ s) & 0x80) != 0);
        setf(FC, s > 0xFF);
        m.a = static_cast<u8>(s);
        nz(m.a);
    }
    void cmp(u8 r, u8 v) { setf(FC, r >= v); nz(static_cast<u8>(r - v)); }

    StepOut step() {
        const u16 pc0 = m.pc;
        const u8 op = rd(pc0);
        u32 cyc = 0;
        u16 ea = 0;
        bool cross = false;
        auto imm8 = [&] { return rd(static_cast<u16>(pc0 + 1)); };
        auto a_zp = [&] { ea = imm8(); m.pc = pc0 + 2; };
        auto a_zpx = [&] { ea = static_cast<u8>(imm8() + m.x); m.pc = pc0 + 2; };
        auto a_zpy = [&] { ea = static_cast<u8>(imm8() + m.y); m.pc = pc0 + 2; };
        auto a_abs = [&] { ea = rd16(static_cast<u16>(pc0 + 1)); m.pc = pc0 + 3; };
        auto a_absi = [&](u8 r) {
            const u16 b = rd16(static_cast<u16>(pc0 + 1));
            ea = static_cast<u16>(b + r);
            cross = (b & 0xFF00) != (ea & 0xFF00);
            m.pc = pc0 + 3;
        };
        auto a_indx = [&] {
            const u8 z = static_cast<u8>(imm8() + m.x);
            ea = static_cast<u16>(m.ram[z] | (m.ram[static_cast<u8>(z + 1)] << 8));
            m.pc = pc0 + 2;
        };
        auto a_indy = [&] {
            const u8 z = imm8();
            const u16 b = static_cast<u16>(m.ram[z] | (m.ram[static_cast<u8>(z + 1)] << 8));
            ea = static_cast<u16>(b + m.y);
            cross = (b & 0xFF00) != (ea & 0xFF00);
            m.pc = pc0 + 2;
        };
        // read-group address by the standard column layout: mode index -> (setup, base cycles)
        auto read_mode = [&](int mode) -> u8 {
            switch (mode) {
                case 0: a_indx(); cyc = 6; break;
                case 1: a_zp(); cyc = 3; break;
                case 2: m.pc = pc0 + 2; cyc = 2; return imm8();
                case 3: a_abs(); cyc = 4; break;
                case 4: a_indy(); cyc = 5 + (cross ? 1 : 0); break;
                case 5: a_zpx(); cyc = 4; break;
                case 6: a_absi(m.y); cyc = 4 + (cross ? 1 : 0); break;
                default: a_absi(m.x); cyc = 4 + (cross ? 1 : 0); break;
            }
            return rd(ea);
        };
        auto branch = [&](bool take) {
            const int8_t d = static_cast<int8_t>(imm8());
            m.pc = pc0 + 2;
            cyc = 2;
            if (take) {
                const u16 to = static_cast<u16>(m.pc + d);
                cyc += ((to & 0xFF00) != (m.pc & 0xFF00)) ? 2 : 1;
                m.pc = to;
            }
        };
        // read-modify-write on memory: modes zp/zpx/abs/absx
        auto rmw_addr = [&](u8 opc) {
            switch ((opc >> 2) & 7) {
                case 1: a_zp(); cyc = 5; break;
                case 3: a_abs(); cyc = 6; break;
                case 5: a_zpx(); cyc = 6; break;
                default: a_absi(m.x); cyc = 7; break;
            }
        };
        switch (op) {
            // ---- loads / stores
            case 0xA9: case 0xA5: case 0xB5: case 0xAD: case 0xBD: case 0xB9: case 0xA1: case 0xB1:
                m.a = read_mode((op >> 2) & 7); nz(m.a); break;
            case 0xA2: m.x = imm8(); m.pc = pc0 + 2; cyc = 2; nz(m.x); break;
            case 0xA6: a_zp(); cyc = 3; m.x = rd(ea); nz(m.x); break;
            case 0xB6: a_zpy(); cyc = 4; m.x = rd(ea); nz(m.x); break;
            case 0xAE: a_abs(); cyc = 4; m.x = rd(ea); nz(m.x); break;
            case 0xBE: a_absi(m.y); cyc = 4 + (cross ? 1 : 0); m.x = rd(ea); nz(m.x); break;
            case 0xA0: m.y = imm8(); m.pc = pc0 + 2; cyc = 2; nz(m.y); break;
            case 0xA4: a_zp(); cyc = 3; m.y = rd(ea); nz(m.y); break;
            case 0xB4: a_zpx(); cyc = 4; m.y = rd(ea); nz(m.y); break;
            case 0xAC: a_abs(); cyc = 4; m.y = rd(ea); nz(m.y); break;
            case 0xBC: a_absi(m.x); cyc = 4 + (cross ? 1 : 0); m.y = rd(ea); nz(m.y); break;
            case 0x85: a_zp(); cyc = 3; wr(ea, m.a); break;
            case 0x95: a_zpx(); cyc = 4; wr(ea, m.a); break;
            case 0x8D: a_abs(); cyc = 4; wr(ea, m.a); break;
            case 0x9D: a_absi(m.x); cyc = 5; wr(ea, m.a); break;
            case 0x99: a_absi(m.y); cyc = 5; wr(ea, m.a); break;
            case 0x81: a_indx(); cyc = 6; wr(ea, m.a); break;
            case 0x91: a_indy(); cyc = 6; wr(ea, m.a); break;
            case 0x86: a_zp(); cyc = 3; wr(ea, m.x); break;
            case 0x96: a_zpy(); cyc = 4; wr(ea, m.x); break;
            case 0x8E: a_abs(); cyc = 4; wr(ea, m.x); break;
            case 0x84: a_zp(); cyc = 3; wr(ea, m.y); break;
            case 0x94: a_zpx(); cyc = 4; wr(ea, m.y); break;
            case 0x8C: a_abs(); cyc = 4; wr(ea, m.y); break;
            // ---- ALU group
            case 0x69: case 0x65: case 0x75: case 0x6D: case 0x7D: case 0x79: case 0x61: case 0x71:
                adc(read_mode((op >> 2) & 7)); break;
            case 0xE9: case 0xE5: case 0xF5: case 0xED: case 0xFD: case 0xF9: case 0xE1: case 0xF1:
                adc(static_cast<u8>(read_mode((op >> 2) & 7) ^ 0xFF)); break;
            case 0x29: case 0x25: case 0x35: case 0x2D: case 0x3D: case 0x39: case 0x21: case 0x31:
                m.a &= read_mode((op >> 2) & 7); nz(m.a); break;
            case 0x09: case 0x05: case 0x15: case 0x0D: case 0x1D: case 0x19: case 0x01: case 0x11:
                m.a |= read_mode((op >> 2) & 7); nz(m.a); break;
            case 0x49: case 0x45: case 0x55: case 0x4D: case 0x5D: case 0x59: case 0x41: case 0x51:
                m.a ^= read_mode((op >> 2) & 7); nz(m.a); break;
            case 0xC9: case 0xC5: case 0xD5: case 0xCD: case 0xDD: case 0xD9: case 0xC1: case 0xD1:
                cmp(m.a, read_mode((op >> 2) & 7)); break;
            case 0xE0: cmp(m.x, imm8()); m.pc = pc0 + 2; cyc = 2; break;
            case 0xE4: a_zp(); cyc = 3; cmp(m.x, rd(ea)); break;
            case 0xEC: a_abs(); cyc = 4; cmp(m.x, rd(ea)); break;
            case 0xC0: cmp(m.y, imm8()); m.pc = pc0 + 2; cyc = 2; break;
            case 0xC4: a_zp(); cyc = 3; cmp(m.y, rd(ea)); break;
            case 0xCC: a_abs(); cyc = 4; cmp(m.y, rd(ea)); break;
            case 0x24: case 0x2C: {
                if (op == 0x24) { a_zp(); cyc = 3; } else { a_abs(); cyc = 4; }
                const u8 v = rd(ea);
                setf(FZ, (m.a & v) == 0);
                m.p = static_cast<u8>((m.p & 0x3F) | (v & 0xC0));
                break;
            }
            // ---- shifts / inc / dec
            case 0x0A: setf(FC, m.a & 0x80); m.a = static_cast<u8>(m.a << 1); nz(m.a); m.pc = pc0 + 1; cyc = 2; break;
            case 0x4A: setf(FC, m.a & 1); m.a >>= 1; nz(m.a); m.pc = pc0 + 1; cyc = 2; break;
            case 0x2A: { const u8 cin = m.p & FC; setf(FC, m.a & 0x80); m.a = static_cast<u8>((m.a << 1) | cin); nz(m.a); m.pc = pc0 + 1; cyc = 2; break; }
            case 0x6A: { const u8 cin = m.p & FC; setf(FC, m.a & 1); m.a = static_cast<u8>((m.a >> 1) | (cin << 7)); nz(m.a); m.pc = pc0 + 1; cyc = 2; break; }
            case 0x06: case 0x16: case 0x0E: case 0x1E:
            case 0x46: case 0x56: case 0x4E: case 0x5E:
            case 0x26: case 0x36: case 0x2E: case 0x3E:
            case 0x66: case 0x76: case 0x6E: case 0x7E:
            case 0xC6: case 0xD6: case 0xCE: case 0xDE:
            case 0xE6: case 0xF6: case 0xEE: case 0xFE: {
                rmw_addr(op);
                u8 v = rd(ea);
                const u8 cin = m.p & FC;
                switch (op >> 5) {
                    case 0: setf(FC, v & 0x80); v = static_cast<u8>(v << 1); break;             // ASL
                    case 1: setf(FC, v & 0x80); v = static_cast<u8>((v << 1) | cin); break;     // ROL
                    case 2: setf(FC, v & 1); v >>= 1; break;                                     // LSR
                    case 3: setf(FC, v & 1); v = static_cast<u8>((v >> 1) | (cin << 7)); break;  // ROR
                    case 6: v = static_cast<u8>(v - 1); break;                                   // DEC
                    default: v = static_cast<u8>(v + 1); break;                                  // INC
                }
                nz(v);
                wr(ea, v);
                break;
            }
            case 0xCA: --m.x; nz(m.x); m.pc = pc0 + 1; cyc = 2; break;
            case 0x88: --m.y; nz(m.y); m.pc = pc0 + 1; cyc = 2; break;
            case 0xE8: ++m.x; nz(m.x); m.pc = pc0 + 1; cyc = 2; break;
            case 0xC8: ++m.y; nz(m.y); m.pc = pc0 + 1; cyc = 2; break;
            // ---- transfers / flags
            case 0xAA: m.x = m.a; nz(m.x); m.pc = pc0 + 1; cyc = 2; break;
            case 0xA8: m.y = m.a; nz(m.y); m.pc = pc0 + 1; cyc = 2; break;
            case 0xBA: m.x = m.sp; nz(m.x); m.pc = pc0 + 1; cyc = 2; break;
            case 0x8A: m.a = m.x; nz(m.a); m.pc = pc0 + 1; cyc = 2; break;
            case 0x9A: m.sp = m.x; m.pc = pc0 + 1; cyc = 2; break;
            case 0x98: m.a = m.y; nz(m.a); m.pc = pc0 + 1; cyc = 2; break;
            case 0x18: setf(FC, false); m.pc = pc0 + 1; cyc = 2; break;
            case 0x38: setf(FC, true); m.pc = pc0 + 1; cyc = 2; break;
            case 0x58: setf(FI, false); m.pc = pc0 + 1; cyc = 2; break;
            case 0x78: setf(FI, true); m.pc = pc0 + 1; cyc = 2; break;
            case 0xB8: setf(FV, false); m.pc = pc0 + 1; cyc = 2; break;
            case 0xD8: setf(FD, false); m.pc = pc0 + 1; cyc = 2; break;
            case 0xF8: setf(FD, true); m.pc = pc0 + 1; cyc = 2; break;
            case 0xEA: m.pc = pc0 + 1; cyc = 2; break;
            // ---- stack
            case 0x48: push(m.a); m.pc = pc0 + 1; cyc = 3; break;
            case 0x08: push(static_cast<u8>(m.p | FB | FU)); m.pc = pc0 + 1; cyc = 3; break;
            case 0x68: m.a = pull(); nz(m.a); m.pc = pc0 + 1; cyc = 4; break;
            case 0x28: m.p = static_cast<u8>((pull() & ~FB) | FU); m.pc = pc0 + 1; cyc = 4; break;
            // ---- control
            case 0x4C: m.pc = rd16(static_cast<u16>(pc0 + 1)); cyc = 3; break;
            case 0x6C: {
                const u16 ptr = rd16(static_cast<u16>(pc0 + 1));
                const u16 hi = static_cast<u16>((ptr & 0xFF00) | ((ptr + 1) & 0xFF));
                m.pc = static_cast<u16>(rd(ptr) | (rd(hi) << 8));
                cyc = 5;
                break;
            }
            case 0x20: {
                const u16 to = rd16(static_cast<u16>(pc0 + 1));
                const u16 ret = static_cast<u16>(pc0 + 2);
                push(static_cast<u8>(ret >> 8));
                push(static_cast<u8>(ret));
                m.pc = to;
                cyc = 6;
                break;
            }
            case 0x60: { const u8 lo = pull(); const u8 hi = pull(); m.pc = static_cast<u16>(((hi << 8) | lo) + 1); cyc = 6; break; }
            case 0x40: {
                m.p = static_cast<u8>((pull() & ~FB) | FU);
                const u8 lo = pull(); const u8 hi = pull();
                m.pc = static_cast<u16>((hi << 8) | lo);
                cyc = 6;
                break;
            }
            case 0x00: {
                const u16 ret = static_cast<u16>(pc0 + 2);
                push(static_cast<u8>(ret >> 8));
                push(static_cast<u8>(ret));
                push(static_cast<u8>(m.p | FB | FU));
                m.p |= FI;
                m.pc = rd16(0xFFFE);
                cyc = 7;
                break;
            }
            case 0x90: branch(!(m.p & FC)); break;
            case 0xB0: branch(m.p & FC); break;
            case 0xF0: branch(m.p & FZ); break;
            case 0xD0: branch(!(m.p & FZ)); break;
            case 0x30: branch(m.p & FN); break;
            case 0x10: branch(!(m.p & FN)); break;
            case 0x50: branch(!(m.p & FV)); break;
            case 0x70: branch(m.p & FV); break;
            default:
                m.pc = pc0;
                return StepOut{0, op, pc0, true};
        }
        m.cycles += cyc;
        return StepOut{cyc, op, pc0, false};
    }
};

// ------------------------------------------------------------------------------------------------ console step

struct ConsoleStep { StepOut cpu; u32 ppu_cycles; };

// One instruction with the PPU settled lazily (patch:834-861 restated, with the unpinned base parts defined here):
// NMI / level IRQ entry, the instruction, OAM DMA stall (513 + odd-cycle), DMC fetch steals.
inline ConsoleStep console_step(const Cart& c, Console& m, u32 pending) {
    Cpu cpu{c, m};
    const u64 before = m.cycles;
    if (m.nmi_pending) {
        m.nmi_pending = 0;
        cpu.interrupt(0xFFFA);
    } else if (c.board == kMmc3 && m.irq_line && !(m.p & FI)) {
        cpu.interrupt(0xFFFE);
    }
    m.now = m.frame_dot + pending + static_cast<u32>(m.cycles - before) * 3;
    const u16 logged = m.log_count;
    const StepOut s = cpu.step();
    if (s.illegal) return ConsoleStep{s, 0};
    if (m.log_count != logged) log_set_cycles(m, logged, s.cycles);
    if (m.dma_pending) {
        m.dma_pending = 0;
        m.cycles += 513 + (m.cycles & 1);
    }
    if (m.cycles >= m.dmc_event) m.cycles += dmc_service(m, m.cycles, true);
    return ConsoleStep{s, static_cast<u32>(m.cycles - before) * 3};
}

// Skip a JMP-to-self loop up to the next PPU event (patch:882-893 restated).
inline void fast_forward_idle(const Cart& c, Console& m) {
    if (m.nmi_pending) return;
    const u32 to_event = dots_to_event(c, m);
    const u32 jumps = (to_event + 8) / 9;
    if (jumps == 0) return;
    const u32 cpu_cycles = jumps * 3;
    m.cycles += cpu_cycles;
    if (m.cycles >= m.dmc_event) (void)dmc_service(m, m.cycles, false);
    ppu_settle(c, m, cpu_cycles * 3);
}

constexpr u64 kBudget = 200000;   // instructions per frame (rl/csrc/nes_machine.cuh:30)

// Run until absolute PPU dot `target` (rl/csrc/nes_machine.cuh:67-103). Returns pc << 8 | opcode on a fault.
inline u32 step_until(const Cart& c, Console& m, u64 target) {
    u64 instructions = 0;
    u32 fault = 0;
    u32 pending = 0;
    u32 to_event = dots_to_event(c, m);
    bool done = false;
    auto reached = [&] { return m.frame * kFrameDots + m.frame_dot >= target; };
    while (instructions < kBudget && !done) {
        if (pending >= to_event) {
            ppu_settle(c, m, pending);
            pending = 0;
            to_event = dots_to_event(c, m);
            if (reached()) break;
        }
        const ConsoleStep st = console_step(c, m, pending);
        if (st.cpu.illegal) { fault = (u32(st.cpu.pc) << 8) | st.cpu.opcode; break; }
        pending += st.ppu_cycles;
        ++instructions;
        if (st.cpu.opcode == 0x4C && m.pc == st.cpu.pc) {
            ppu_settle(c, m, pending);
            pending = 0;
            if (reached()) break;
            fast_forward_idle(c, m);
            to_event = dots_to_event(c, m);
            done = reached();
        }
    }
    if (pending != 0) ppu_settle(c, m, pending);
    return fault;
}

// Power-on (NeSLE cold_reset_console_env, base absent; restated, patch:2755-2777 adds DMC, sprite-0, frame log).
inline void cold_reset(const Cart& c, Console& m) {
    std::memset(&m, 0, sizeof m);
    m.prg_bank = 0;
    if (board_paged(c.board)) board::power_on(c, m);
    m.sp = 0xFD;
    m.p = 0x24;
    m.cycles = 7;
    dmc_reset(m, 7);
    m.pc = static_cast<u16>(read_prg(c, m, 0xFFFC) | (read_prg(c, m, 0xFFFD) << 8));
    log_reset(c, m);
    std::memset(m.ram, 0xFF, sizeof m.ram);   // fceumm power-on RAM (rl/csrc/rlenv_build.hpp:86)
    m.frame_dot = 0;
}

}  // namespace orc
