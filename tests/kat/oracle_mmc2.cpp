// TEST INFRASTRUCTURE: MMC2 (mapper 9) in the CPU oracle (oracle/nes.hpp) against the behaviour the reference's
// patch gives the board; the reference has no test of its own for it, so these checks follow its code:
//   * registers $A000-$F000 and the page tables: third_party/nesle-extensions.patch:3147-3156, 3027-3035,
//   * power-on latches ($FE, $FE): patch:3080-3082,
//   * the latch hook on CPU-driven PPU addresses ($2006 second write, $2007 before its buffer refill and after its
//     increment) and the $0FD0-$0FEF / $1FD0-$1FEF ranges: patch:615-636, 674-760, 3195-3222,
//   * frame-log events for latch and CHR-register changes while a frame is drawn: patch:615-665,
//   * the replay's hook on fetched pattern addresses: patch:1385-1402.
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

struct Board {
    Cart c;
    Console m{};
    Board() {
        c.board = kMmc2;
        c.arrangement = 0;
        c.prg.assign(128 * 1024, 0);
        c.chr.resize(128 * 1024);
        for (std::size_t i = 0; i < c.chr.size(); ++i) c.chr[i] = static_cast<u8>(i >> 12);   // byte = its 4 KB bank
        c.prg_page_mask = 15;
        c.chr_page_mask = 127;
        board::power_on(c, m);
    }
    void wr(u16 a, u8 v) { cpu_write(c, m, a, v); }
    u8 rd(u16 a) { return cpu_read(c, m, a); }
    void addr(u16 a) { wr(0x2006, static_cast<u8>(a >> 8)); wr(0x2006, static_cast<u8>(a)); }
    u32 half_bank(u32 half) const { return (m.chr_page[4 * half] >> 10) / 4; }
    bool logged(u8 kind, u32 value, u32 aux) const {
        const u32* bank = log_bank_ptr(m, (m.log_bank & 1u) ^ 1u);
        for (u32 i = 0; i < m.log_count && i < kLogEvents; ++i) {
            const u32 w0 = bank[kLogHeader + 2 * i], w1 = bank[kLogHeader + 2 * i + 1];
            if ((w0 >> 24) == kind && (w1 & 0xFF) == value && ((w1 >> 8) & 0xFF) == aux) return true;
        }
        return false;
    }
};

void registers_and_pages() {
    Board b;
    CHECK(b.m.regs[board::kMmc2Latch0] == 1 && b.m.regs[board::kMmc2Latch1] == 1);
    b.wr(0xB000, 5); b.wr(0xC000, 9); b.wr(0xD000, 17); b.wr(0xE000, 0x3E);   // $E000 keeps 5 bits: 30
    b.wr(0xA000, 0x13);                                                         // PRG keeps 4 bits: 3
    CHECK(b.m.regs[3] == 30 && b.m.regs[board::kMmc2Prg] == 3);
    CHECK(b.m.prg_page[0] == (3u << 13) && b.m.prg_page[1] == (13u << 13) && b.m.prg_page[2] == (14u << 13) &&
          b.m.prg_page[3] == (15u << 13));
    CHECK(b.half_bank(0) == 9 && b.half_bank(1) == 30);      // both halves on their $FE register
    for (u32 i = 0; i < 4; ++i) CHECK(b.m.chr_page[i] == ((4 * 9 + i) << 10));
    b.wr(0xF000, 0); CHECK(b.m.mirroring == kPageVertical);
    b.wr(0xF000, 1); CHECK(b.m.mirroring == kPageHorizontal);
    b.wr(0x9FFF, 0x1F); CHECK(b.m.regs[0] == 5 && b.half_bank(0) == 9);   // $8000-$9FFF: no register
}

void cpu_address_hook() {
    Board b;
    b.wr(0xB000, 5); b.wr(0xC000, 9); b.wr(0xD000, 17); b.wr(0xE000, 30);
    b.addr(0x0FD8); CHECK(b.m.regs[board::kMmc2Latch0] == 0 && b.half_bank(0) == 5);
    b.addr(0x1FE8); CHECK(b.m.regs[board::kMmc2Latch1] == 1 && b.half_bank(1) == 30);
    b.addr(0x1FD0); CHECK(b.m.regs[board::kMmc2Latch1] == 0 && b.half_bank(1) == 17);
    b.addr(0x0FC8); CHECK(b.m.regs[board::kMmc2Latch0] == 0);   // outside $0FD0-$0FEF: no change
    b.addr(0x2FE0); CHECK(b.m.regs[board::kMmc2Latch0] == 0 && b.m.regs[board::kMmc2Latch1] == 0);
    // $2007 reads: the buffer refills through the bank the address picks, so the second read returns its byte
    b.addr(0x0FD0);
    (void)b.rd(0x2007);
    CHECK(b.rd(0x2007) == 5);
    b.addr(0x0FE8);                       // latch 0 -> $FE (bank 9); the buffer still holds a bank-5 byte
    CHECK(b.rd(0x2007) == 5);
    CHECK(b.rd(0x2007) == 9);
    // a $2007 write moves v and the hook sees the new address
    b.addr(0x0FDF);                       // latch 0 -> $FD
    b.wr(0x2007, 0);                      // CHR ROM: ignored; v -> $0FE0: latch 0 -> $FE
    CHECK(b.m.regs[board::kMmc2Latch0] == 1 && b.half_bank(0) == 9);
}

void logged_while_drawn() {
    Board b;
    b.wr(0xB000, 5); b.wr(0xC000, 9);
    b.m.now = 100 * kDots;                // inside the picture: the frame log takes events
    b.addr(0x0FD8);
    CHECK(b.logged(kEvMmc2, 0, board::kMmc2Latch0));
    b.addr(0x0FE8);
    CHECK(b.logged(kEvMmc2, 1, board::kMmc2Latch0));
    b.wr(0xC000, 11);                     // the $FE register of the half now on $FE: pages and register logged
    CHECK(b.logged(kEvMmc2, 11, 1));
    CHECK(b.logged(kEvChr, 4 * 11, 0) && b.logged(kEvChr, 4 * 11 + 3, 3));
    const u32 n = b.m.log_count;
    b.addr(0x0FE8);                       // no change: nothing more than the two address writes
    CHECK(b.m.log_count == n + 2);
}

void replay_hook() {
    Board b;
    b.wr(0xD000, 17); b.wr(0xE000, 30);
    u32 h[kLogBank] = {};
    fill_header(b.c, b.m, 0, 0x18, h);
    const Src src = make_src(b.c, b.m, h, 0, b.m.nt, b.m.oam);
    RState s;
    r_load(s, h);
    CHECK(s.latch[1] == 1 && s.creg[3] == 30);
    r_mmc2_hook(src, s, 0x1FD7);          // a $1FD0-$1FDF fetch: half 1 on its $FD register
    CHECK(s.latch[1] == 0 && s.chr[4] == 4 * 17 && s.chr[7] == 4 * 17 + 3);
    r_mmc2_hook(src, s, 0x1FF0);          // $1FF0: outside the ranges
    CHECK(s.latch[1] == 0);
    r_mmc2_hook(src, s, 0x1FE3);
    CHECK(s.latch[1] == 1 && s.chr[4] == 4 * 30);
}

}  // namespace

int main() {
    registers_and_pages();
    cpu_address_hook();
    logged_while_drawn();
    replay_hook();
    if (g_failed) {
        std::printf("%d MMC2 checks failed\n", g_failed);
        return 1;
    }
    std::printf("all MMC2 checks passed\n");
    return 0;
}
