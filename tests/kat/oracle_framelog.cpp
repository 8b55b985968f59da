// TEST INFRASTRUCTURE: the frame log in the CPU oracle (oracle/nes.hpp) against the patch's recording code, which
// every picture depends on and which the reference's tests do not cover directly:
//   * events: one per PPU register write while a frame is drawn (PPU dot 17 bits | kind << 24; value | aux << 8),
//     scroll / address writes with the write toggle in aux, palette writes with their index, nothing in vblank,
//     a run of $2007 writes with rendering off merged into one event (repeat count in aux, up to 256), the overflow
//     bit past 256 events, the instruction's cycles stamped afterwards: patch:982-999, 1157-1185,
//   * FCEUmm's time base (dot offset 11, the pre-render line as negative time, short frames): patch:951-965,
//   * the frame's emphasis tint (the most frequent emphasis among lines 0-239 of the last $2001 write that had any;
//     none: the previous tint): patch:1065-1099.
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
        log_reset(c, m);
    }
    void wr(u16 a, u8 v) { cpu_write(c, m, a, v); }
    const u32* bank() const { return log_bank_ptr(m, (m.log_bank & 1u) ^ 1u); }
    u32 kind(u32 i) const { return bank()[kLogHeader + 2 * i] >> 24; }
    u32 dot(u32 i) const { return bank()[kLogHeader + 2 * i] & 0x1FFFFu; }
    u32 cyc(u32 i) const { return (bank()[kLogHeader + 2 * i] >> 17) & 0xFu; }
    u32 value(u32 i) const { return bank()[kLogHeader + 2 * i + 1] & 0xFFu; }
    u32 aux(u32 i) const { return (bank()[kLogHeader + 2 * i + 1] >> 8) & 0xFFu; }
};

void events() {
    Nes n;
    n.m.now = 50 * kDots + 100;
    n.wr(0x2000, 0x90);
    n.wr(0x2001, 0x1E);
    n.wr(0x2005, 0x10); n.wr(0x2005, 0x20);
    n.wr(0x2006, 0x21); n.wr(0x2006, 0x00);
    n.wr(0x2007, 5); n.wr(0x2007, 6);                       // rendering on: one event per write
    n.wr(0x2006, 0x3F); n.wr(0x2006, 0x11);
    n.wr(0x2007, 0x2A);                                     // palette entry $11
    CHECK(n.m.log_count == 11);
    CHECK(n.kind(0) == kEvCtrl && n.value(0) == 0x90 && n.dot(0) == 50 * kDots + 100);
    CHECK(n.kind(1) == kEvMask && n.value(1) == 0x1E);
    CHECK(n.kind(2) == kEvScroll && n.value(2) == 0x10 && n.aux(2) == 0);
    CHECK(n.kind(3) == kEvScroll && n.value(3) == 0x20 && n.aux(3) == 1);
    CHECK(n.kind(4) == kEvAddr && n.aux(4) == 0 && n.kind(5) == kEvAddr && n.aux(5) == 1 && n.value(5) == 0x00);
    CHECK(n.kind(6) == kEvDataWrite && n.kind(7) == kEvDataWrite && n.aux(6) == 0 && n.aux(7) == 0);
    CHECK(n.kind(10) == kEvPalette && n.value(10) == 0x2A && n.aux(10) == 0x11);
    log_set_cycles(n.m, 9, 22);                             // the instruction's cycles, capped at 15
    CHECK(n.cyc(8) == 0 && n.cyc(9) == 15 && n.cyc(10) == 15);
    // rendering off: a VRAM upload is one event per 256 writes
    n.wr(0x2001, 0x00);
    n.wr(0x2006, 0x20); n.wr(0x2006, 0x00);
    const u32 before = n.m.log_count;
    for (int i = 0; i < 300; ++i) n.wr(0x2007, static_cast<u8>(i));
    CHECK(n.m.log_count == before + 2);
    CHECK(n.kind(before) == kEvDataWrite && n.aux(before) == 0xFF && n.aux(before + 1) == 300 - 256 - 1);
    // vblank: nothing is logged
    n.m.now = kVblankDot + 5;
    const u32 at_vblank = n.m.log_count;
    n.wr(0x2000, 0x10); n.wr(0x2001, 0x1E);
    CHECK(n.m.log_count == at_vblank);
    // past 256 events the bank is marked overflowed
    n.m.now = 100 * kDots;
    for (int i = 0; i < 300; ++i) n.wr(0x2000, static_cast<u8>(i));
    CHECK(n.m.log_count == kLogEvents && (n.bank()[0] & kLogOverflow) != 0);
}

void time_base() {
    CHECK(fceumm_time(0, 0) == 11 && fceumm_time(100 * kDots, 0) == 100 * 341 + 11);
    CHECK(fceumm_time(kPreRenderDot, 0) == static_cast<int>(kPreRenderDot) - static_cast<int>(kFrameDots) + 11);
    CHECK(fceumm_time(kPreRenderDot, 1) == fceumm_time(kPreRenderDot, 0) + 1);   // the short frame's missing dot
    CHECK(nesle_dot(fceumm_time(5000, 0)) == 5000u);
}

u32 emphasis_of(u8 header_mask, std::vector<std::pair<int, u8>> mask_writes, u32 previous) {
    // a header with mask `header_mask` and $2001 writes at FCEUmm times (first, value)
    std::vector<u32> h(kLogBank, 0);
    h[1] = static_cast<u32>(header_mask) << 8;
    u32 n = 0;
    for (const auto& w : mask_writes) {
        h[kLogHeader + 2 * n] = (nesle_dot(w.first) & 0x1FFFFu) | (static_cast<u32>(kEvMask) << 24);
        h[kLogHeader + 2 * n + 1] = w.second;
        ++n;
    }
    h[0] = n;
    return log_emphasis(h.data(), previous);
}

void emphasis() {
    CHECK(emphasis_of(0x1E, {}, 5) == 5);                               // none: the previous tint
    CHECK(emphasis_of(0x3E, {}, 5) == 1);                               // red on every line
    CHECK(emphasis_of(0x3E, {{100 * 341 - 1, 0x5E}}, 0) == 2);          // 100 lines red, 140 green
    CHECK(emphasis_of(0x3E, {{120 * 341 - 1, 0x5E}}, 0) == 1);          // 120 / 120: the lower wins
    CHECK(emphasis_of(0x5E, {{10 * 341, 0x1E}}, 0) == 2);               // a write without emphasis changes nothing
    CHECK(emphasis_of(0xFE, {}, 3) == 3);                               // all three bits: not a tint
    CHECK(emphasis_of(0x1E, {{-5, 0x9E}}, 0) == 4);                     // set before line 0 (pre-render time)
}

}  // namespace

int main() {
    events();
    time_base();
    emphasis();
    if (g_failed) {
        std::printf("%d frame-log checks failed\n", g_failed);
        return 1;
    }
    std::printf("all frame-log checks passed\n");
    return 0;
}
