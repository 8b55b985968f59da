// TEST INFRASTRUCTURE: the PPU's timing events in the CPU oracle (oracle/nes.hpp) against the patch's step code:
//   * $2002's vblank flag 12 dots before the vblank dot, NMI at the vblank dot, the flag and the sprite-0 bit cleared
//     12 dots before the pre-render dot, the frame log frozen at vblank and captured at pre-render, sprite 0's
//     evaluation scheduled at dot (y + 1) * 341 - 20 of the next frame: patch:1964-1972, 2150-2232,
//   * the sprite-0 hit's dot: the line pixel at which FCEUmm's RefreshLine first sees it, 12 dots before the
//     instruction end that reads it: patch:1740-1789.
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
    Nes() {
        c.board = kNrom;
        c.arrangement = 0;
        c.prg.assign(32768, 0);
        c.chr.assign(8192, 0);
        for (auto& b : m.oam) b = 0xFF;
        log_reset(c, m);
    }
    void to(u32 dot) { ppu_settle(c, m, dot - m.frame_dot); }   // settle forward to frame dot `dot`
};

void vblank_events() {
    Nes n;
    n.m.ctrl = 0x80;
    n.to(kVblankFlagDot - 1);
    CHECK((n.m.status & 0x80) == 0);
    n.to(kVblankFlagDot);
    CHECK((n.m.status & 0x80) != 0 && !n.m.nmi_pending);
    const u8 bank_before = n.m.log_bank;
    n.to(kVblankDot - 1);
    CHECK(!n.m.nmi_pending && n.m.log_bank == bank_before);
    n.to(kVblankDot);
    CHECK(n.m.nmi_pending && ((n.m.log_bank ^ bank_before) & 1u));   // NMI and the frozen frame
    n.m.status |= 0x40;
    n.to(kStatusClearDot - 1);
    CHECK((n.m.status & 0xC0) == 0xC0);
    n.to(kStatusClearDot);
    CHECK((n.m.status & 0xC0) == 0);
}

void capture_and_schedule() {
    Nes n;
    n.m.oam[0] = 100;
    n.m.ctrl = 0x10; n.m.mask = 0x1E;
    n.to(kPreRenderDot - 1);
    CHECK(n.m.sprite0_dot == 0);
    n.to(kPreRenderDot);
    const u32* h = log_bank_ptr(n.m, (n.m.log_bank & 1u) ^ 1u);
    CHECK((h[1] & 0xFFu) == 0x10 && ((h[1] >> 8) & 0xFFu) == 0x1E && n.m.log_count == 0);
    CHECK(n.m.sprite0_dot == (nesle_dot(101 * 341 - 20) | kS0Evaluate));
    Nes low;
    low.m.oam[0] = 239;                   // below the picture: nothing to evaluate
    low.to(kPreRenderDot);
    CHECK(low.m.sprite0_dot == 0);
}

void sprite0_dot() {
    Nes n;
    for (int row = 0; row < 16; ++row) n.c.chr[0x0010 + row] = 0xFF;   // tile 1: every pixel opaque (colour 3)
    n.m.nt[1 * 32 + 2] = 0x01;                                           // under pixels 16-23 of lines 8-15
    n.m.oam[0] = 10; n.m.oam[1] = 1; n.m.oam[2] = 0; n.m.oam[3] = 20;    // sprite 0: tile 1 at x 20, lines 11-18
    n.m.ctrl = 0x00; n.m.mask = 0x1E;
    n.to(kPreRenderDot);                                                 // the frame's log starts here
    const Hit0 hit = sprite0_hit(n.c, n.m);
    CHECK(hit.hit && hit.dot == 3749u);   // line 11, pixel 20, first seen at line pixel 37, 12 dots early
    // no opaque background under it: no hit, and the answer holds until sprite 0's last line
    Nes e;
    for (int row = 0; row < 16; ++row) e.c.chr[0x0010 + row] = 0xFF;
    e.m.oam[0] = 10; e.m.oam[1] = 1; e.m.oam[2] = 0; e.m.oam[3] = 20;
    e.m.ctrl = 0x00; e.m.mask = 0x1E;
    e.to(kPreRenderDot);
    const Hit0 miss = sprite0_hit(e.c, e.m);
    CHECK(!miss.hit && miss.dot == nesle_dot((10 + 1 + 15) * 341 + 256));
}

}  // namespace

int main() {
    vblank_events();
    capture_and_schedule();
    sprite0_dot();
    if (g_failed) {
        std::printf("%d PPU timing checks failed\n", g_failed);
        return 1;
    }
    std::printf("all PPU timing checks passed\n");
    return 0;
}
