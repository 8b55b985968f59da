// TEST INFRASTRUCTURE: the oracle's CPU bus (oracle/nes.hpp cpu_read / cpu_write / console_step) against the NES's
// published register behaviour, in place of NeSLE's base bus, which is not vendored: $2002 clears the vblank flag and
// the write toggle, $2005 / $2006 share that toggle ($2006's second write loads v), $2007 reads go through the read
// buffer except palette reads (which refill it from the nametable underneath), v steps by 1 or 32, the palette's
// $3F10/$14/$18/$1C mirrors, the controller's serial port (strobe, 8 bits low first, then 1s), OAM DMA (256 bytes
// from oam_addr, 513 CPU cycles plus 1 on an odd cycle) and the header's nametable mirroring.
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

struct Nes {
    Cart c;
    Console m{};
    explicit Nes(u8 arrangement = 0) {
        c.board = kNrom;
        c.arrangement = arrangement;
        c.prg.assign(32768, 0);
        c.chr.assign(8192, 0);
        m.now = kVblankDot + 100;   // in vblank: nothing is logged
    }
    void wr(u16 a, u8 v) { cpu_write(c, m, a, v); }
    u8 rd(u16 a) { return cpu_read(c, m, a); }
    void addr(u16 a) { wr(0x2006, static_cast<u8>(a >> 8)); wr(0x2006, static_cast<u8>(a)); }
};

void ppu_registers() {
    Nes n;
    n.m.status = 0xC0;
    n.wr(0x2005, 0x08);                          // first write: the toggle is now set
    CHECK(n.m.w == 1);
    const u8 s = n.rd(0x2002);
    CHECK((s & 0xE0) == 0xC0 && (n.m.status & 0x80) == 0 && (n.m.status & 0x40) != 0 && n.m.w == 0);
    n.addr(0x2345);
    CHECK(n.m.v == 0x2345 && n.m.w == 0);
    n.wr(0x2006, 0x7F); n.wr(0x2006, 0xFF);     // the high write keeps 6 bits
    CHECK(n.m.v == 0x3FFF);
    // $2007: nametable reads lag one read behind through the buffer
    n.addr(0x2000);
    n.wr(0x2007, 0x11); n.wr(0x2007, 0x22);
    n.addr(0x2000);
    (void)n.rd(0x2007);
    CHECK(n.rd(0x2007) == 0x11 && n.rd(0x2007) == 0x22);
    // palette reads are immediate and refill the buffer from the nametable underneath ($3F00 -> $2F00)
    n.addr(0x2F00); n.wr(0x2007, 0x5A);
    n.addr(0x3F00); n.wr(0x2007, 0x0F);
    n.addr(0x3F00);
    CHECK(n.rd(0x2007) == 0x0F && n.m.read_buffer == 0x5A);
    // v steps by 32 with control bit 2
    n.wr(0x2000, 0x04);
    n.addr(0x2000);
    n.wr(0x2007, 1);
    CHECK(n.m.v == 0x2020);
    // $3F10 / $14 / $18 / $1C mirror $3F00 / $04 / $08 / $0C
    n.wr(0x2000, 0x00);
    n.addr(0x3F10); n.wr(0x2007, 0x21);
    n.addr(0x3F1C); n.wr(0x2007, 0x2C);
    CHECK(n.m.pal[0x00] == 0x21 && n.m.pal[0x0C] == 0x2C && n.m.pal[0x10] == 0);
    n.addr(0x3F11); n.wr(0x2007, 0x31);
    CHECK(n.m.pal[0x11] == 0x31);               // $3F11 is its own entry
}

void controller() {
    Nes n;
    n.m.pad = 0x29;                              // 0b00101001
    n.wr(0x4016, 1); n.wr(0x4016, 0);
    u32 bits = 0;
    for (int i = 0; i < 8; ++i) bits |= (n.rd(0x4016) & 1u) << i;
    CHECK(bits == 0x29);
    CHECK((n.rd(0x4016) & 1u) == 1 && (n.rd(0x4016) & 1u) == 1);   // after 8 reads: 1
    n.wr(0x4016, 1);                             // strobe held: always the first bit
    CHECK((n.rd(0x4016) & 1u) == 1 && (n.rd(0x4016) & 1u) == 1);
    n.m.pad = 0x28;
    CHECK((n.rd(0x4016) & 1u) == 0);
}

void oam_dma() {
    for (u64 parity : {0ull, 1ull}) {
        Nes n;
        for (int i = 0; i < 256; ++i) n.m.ram[0x0200 + i] = static_cast<u8>(i ^ 0x5A);
        n.m.oam_addr = 4;
        // STA $4014 at $0300 in RAM, A = 2: 4 cycles, then the DMA stall
        n.m.ram[0x0300] = 0x8D; n.m.ram[0x0301] = 0x14; n.m.ram[0x0302] = 0x40;
        n.m.pc = 0x0300; n.m.a = 0x02;
        n.m.cycles = 1000 + parity;
        const ConsoleStep s = console_step(n.c, n.m, 0);
        const u64 after_sta = 1000 + parity + 4;
        CHECK(n.m.cycles == after_sta + 513 + (after_sta & 1));
        CHECK(s.ppu_cycles == static_cast<u32>(n.m.cycles - 1000 - parity) * 3);
        CHECK(n.m.oam[4] == (0 ^ 0x5A) && n.m.oam[3] == (255 ^ 0x5A) && n.m.oam[255] == (251 ^ 0x5A));
    }
}

void mirroring() {
    Nes v(0), h(1);
    v.addr(0x2000); v.wr(0x2007, 0x77);
    CHECK(v.m.nt[nt_offset(v.c, v.m, 0x2800)] == 0x77 && v.m.nt[nt_offset(v.c, v.m, 0x2400)] != 0x77);
    h.addr(0x2000); h.wr(0x2007, 0x66);
    CHECK(h.m.nt[nt_offset(h.c, h.m, 0x2400)] == 0x66 && h.m.nt[nt_offset(h.c, h.m, 0x2800)] != 0x66);
    v.addr(0x3005); v.wr(0x2007, 0x44);         // $3000-$3EFF mirror $2000-$2EFF
    CHECK(v.m.nt[nt_offset(v.c, v.m, 0x2005)] == 0x44);
}

}  // namespace

int main() {
    ppu_registers();
    controller();
    oam_dma();
    mirroring();
    if (g_failed) {
        std::printf("%d bus checks failed\n", g_failed);
        return 1;
    }
    std::printf("all bus checks passed\n");
    return 0;
}
