// TEST INFRASTRUCTURE: the paged boards MMC1, CNROM and MMC3 in the CPU oracle (oracle/nes.hpp) against the board
// code of the reference's patch, which its own tests cover only for the MMC3 page tables (restated in
// oracle_kat.cpp):
//   * MMC1's serial port (reset bit, five LSB-first writes, the register picked by the fifth write's address), its
//     PRG modes, CHR modes, mirroring and PRG-RAM disable: third_party/nesle-extensions.patch:3123-3140, 2995-3019,
//   * CNROM's bank latch (an iNES 1.0 image declares no bus conflicts): patch:3124-3127, 2982-2990,
//   * MMC3's counter, revision B (reload when zero or asked, else decrement; the IRQ line when zero and enabled;
//     $E000 disables and acknowledges): patch:3148-3175, and when it is clocked: dot 266 of each visible line and 256
//     of the pre-render line, while background or sprites are on, unless (ctrl & 0x38) == 0x18: patch:1861-1931.
//   * UxROM (NeSLE's base, not vendored; the published board): the 16 KB bank at $8000 picked by a write, the last
//     16 KB fixed at $C000,
//   * the cold reset: PC from the reset vector, SP $FD, I set, 7 cycles (the published 6502 reset sequence), RAM $FF
//     (rl/csrc/rlenv_build.hpp:86).
// Built and run by tests/test_oracle_kats.py; prints one line per failed check and exits non-zero on any.
#include <cstdio>
#include <vector>

#include "nes.hpp"

namespace {

int g_failed = 0;

#define CHECK(cond)                                                                \
    do {                                                                           \
        if (!(cond)) {                                                             \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);            \
            ++g_failed;                                                            \
        }                                                                          \
    } while (0)

using namespace orc;

struct Paged {
    Cart c;
    Console m{};
    Paged(Board b, u32 prg_kb, u32 chr_kb) {
        c.board = b;
        c.arrangement = 0;
        c.prg.assign(prg_kb * 1024, 0);
        c.chr.assign(chr_kb * 1024, 0);
        c.prg_page_mask = prg_kb / 8 - 1;
        c.chr_page_mask = chr_kb - 1;
        board::power_on(c, m);
    }
    void wr(u16 a, u8 v) { cpu_write(c, m, a, v); }
    void mmc1(u16 a, u8 v) { for (int i = 0; i < 5; ++i) wr(a, static_cast<u8>(v >> i)); }   // LSB first
};

void mmc1() {
    Paged p(kMmc1, 256, 128);
    CHECK(p.m.regs[board::kMmc1Control] == 0x0C);
    // power-on: PRG mode 3, the last 16 KB fixed at $C000
    CHECK(p.m.prg_page[2] == (30u << 13) && p.m.prg_page[3] == (31u << 13));
    p.mmc1(0xE000, 0x05);                           // PRG bank 5 at $8000
    CHECK(p.m.prg_page[0] == (10u << 13) && p.m.prg_page[1] == (11u << 13) && p.m.prg_page[2] == (30u << 13));
    // four writes change nothing; a reset write clears the half-filled shift register
    for (int i = 0; i < 4; ++i) p.wr(0xE000, 1);
    CHECK(p.m.prg_page[0] == (10u << 13));
    p.wr(0x8000, 0x80);
    CHECK(p.m.regs[board::kMmc1Shift] == 0 && p.m.regs[board::kMmc1Count] == 0);
    p.mmc1(0xE000, 0x03);
    CHECK(p.m.prg_page[0] == (6u << 13));
    p.mmc1(0x8000, 0x08 | 0x02);                    // PRG mode 2: $8000 fixed to the first bank, vertical mirroring
    CHECK(p.m.prg_page[0] == 0 && p.m.prg_page[2] == (6u << 13) && p.m.mirroring == kPageVertical);
    p.mmc1(0x8000, 0x00 | 0x03);                    // PRG mode 0 (32 KB, low bit ignored), horizontal
    CHECK(p.m.prg_page[0] == (4u << 13) && p.m.prg_page[3] == (7u << 13) && p.m.mirroring == kPageHorizontal);
    p.mmc1(0x8000, 0x10 | 0x0C | 0x01);             // CHR 4 KB mode, single-screen high
    p.mmc1(0xA000, 7); p.mmc1(0xC000, 20);
    CHECK(p.m.chr_page[0] == (28u << 10) && p.m.chr_page[4] == (80u << 10) && p.m.mirroring == kPageSingleHigh);
    p.mmc1(0x8000, 0x0C);                           // CHR 8 KB mode: register 1 with its low bit cleared
    CHECK(p.m.chr_page[0] == (24u << 10) && p.m.chr_page[4] == (28u << 10) && p.m.mirroring == kPageSingleLow);
    CHECK(prg_ram_enabled(p.c, p.m));
    p.mmc1(0xE000, 0x10 | 0x03);                    // bit 4 of the PRG register disables the cartridge RAM
    CHECK(!prg_ram_enabled(p.c, p.m) && cpu_read(p.c, p.m, 0x6123) == 0x61);   // open bus: the address high byte
}

void cnrom() {
    Paged p(kCnrom, 32, 32);
    CHECK(p.m.chr_page[0] == 0);
    p.wr(0x8123, 2);
    for (u32 i = 0; i < 8; ++i) CHECK(p.m.chr_page[i] == ((16u + i) << 10));
    p.wr(0xFFFF, 7);                                // 4 banks: the bank number wraps through the page mask
    CHECK(p.m.chr_page[0] == ((56u & 31u) << 10));
    CHECK(p.m.prg_page[0] == 0 && p.m.prg_page[3] == (3u << 13));
}

void mmc3_counter() {
    Paged p(kMmc3, 128, 128);
    p.wr(0xC000, 2);                                // latch 2
    p.wr(0xC001, 0);                                // reload at the next clock
    p.wr(0xE001, 0);                                // enabled
    board::mmc3_clock(p.m); CHECK(p.m.regs[board::kMmc3Counter] == 2 && !p.m.irq_line);
    board::mmc3_clock(p.m); CHECK(p.m.regs[board::kMmc3Counter] == 1 && !p.m.irq_line);
    board::mmc3_clock(p.m); CHECK(p.m.regs[board::kMmc3Counter] == 0 && p.m.irq_line);
    p.wr(0xE000, 0);                                // disable + acknowledge
    CHECK(!p.m.irq_line && !p.m.regs[board::kMmc3Enabled]);
    board::mmc3_clock(p.m); CHECK(p.m.regs[board::kMmc3Counter] == 2);   // zero reloads
    board::mmc3_clock(p.m); board::mmc3_clock(p.m);
    CHECK(p.m.regs[board::kMmc3Counter] == 0 && !p.m.irq_line);          // disabled: no IRQ at zero
    p.wr(0xC000, 0); p.wr(0xE001, 0);               // latch 0: revision B raises the IRQ on every clock
    board::mmc3_clock(p.m); CHECK(p.m.irq_line);
}

void mmc3_clock_timing() {
    Paged p(kMmc3, 128, 128);
    p.wr(0xC000, 200);
    p.m.mask = 0x18;
    p.m.ctrl = 0x08;
    auto clocks = [&](u32 start, u32 end) {         // counter clocks in (start, end]
        p.m.regs[board::kMmc3Counter] = 250;
        p.m.regs[board::kMmc3Reload] = 0;
        clock_mmc3(p.m, start, end);
        return 250u - p.m.regs[board::kMmc3Counter];
    };
    CHECK(clocks(0, 266) == 1 && clocks(0, 265) == 0 && clocks(266, 266 + kDots) == 1);
    CHECK(clocks(0, kFrameDots) == 241);            // 240 visible lines + the pre-render line
    CHECK(clocks(261 * kDots + 255, 261 * kDots + 256) == 1);
    CHECK(clocks(240 * kDots, 261 * kDots) == 0);   // no clock in vblank
    p.m.ctrl = 0x18;                                // both tables at $1000, 8x8 sprites: never clocked
    CHECK(clocks(0, kFrameDots) == 0);
    p.m.ctrl = 0x38;                                // 8x16 sprites: clocked again
    CHECK(clocks(0, kFrameDots) == 241);
    p.m.mask = 0x00;                                // rendering off
    CHECK(clocks(0, kFrameDots) == 0);
    CHECK(dots_to_mmc3_clock(0) == 266 && dots_to_mmc3_clock(266) == kDots &&
          dots_to_mmc3_clock(239 * kDots + 266) == 22 * kDots - 10);
}

void uxrom() {
    Cart c;
    c.board = kUxrom;
    c.arrangement = 0;
    c.prg.resize(128 * 1024);
    for (std::size_t i = 0; i < c.prg.size(); ++i) c.prg[i] = static_cast<u8>(i >> 14);   // byte = its 16 KB bank
    c.chr.assign(8192, 0);
    c.bank_mask = 7;
    c.fixed_base = 128 * 1024 - 16384;
    Console m{};
    cpu_write(c, m, 0x8000, 5);
    CHECK(cpu_read(c, m, 0x8123) == 5 && cpu_read(c, m, 0xBFFF) == 5 && cpu_read(c, m, 0xC000) == 7);
    cpu_write(c, m, 0xFFF0, 0x0B);                  // the bank number keeps the mask's bits
    CHECK(cpu_read(c, m, 0x9000) == 3 && cpu_read(c, m, 0xFFFF) == 7);
}

void cold_reset_state() {
    Cart c;
    c.board = kNrom;
    c.arrangement = 0;
    c.prg.assign(32768, 0);
    c.prg[0x7FFC] = 0x34; c.prg[0x7FFD] = 0x92;    // reset vector $9234
    c.chr.assign(8192, 0);
    Console m;
    cold_reset(c, m);
    CHECK(m.pc == 0x9234 && m.sp == 0xFD && (m.p & FI) && m.p == 0x24 && m.cycles == 7);
    bool ram_ff = true;
    for (u8 b : m.ram) ram_ff = ram_ff && b == 0xFF;
    CHECK(ram_ff && m.frame_dot == 0);
}

}  // namespace

int main() {
    uxrom();
    cold_reset_state();
    mmc1();
    cnrom();
    mmc3_counter();
    mmc3_clock_timing();
    if (g_failed) {
        std::printf("%d board checks failed\n", g_failed);
        return 1;
    }
    std::printf("all board checks passed\n");
    return 0;
}
