// TEST INFRASTRUCTURE: the reference's own known-answer tests for the environment's emulator extensions, restated
// against the CPU oracle (oracle/nes.hpp) so that its DMC and frame-log replay are pinned to the reference's expected
// values, not only to this repository's GPU build. Scenarios and expected values follow
//   * DMC sample channel, $4015 status, stolen CPU cycles: third_party/nesle-extensions.patch:4065-4207
//     (tests/cpp/test_cuda_apu.cpp),
//   * frame-log replay renderer: patch:4355-4522 (tests/cpp/test_cuda_render.cpp). The reference compares the
//     FCEUmm RGB of a palette value; the environment's pictures are the palette values themselves, so the checks
//     here compare those (a stricter test for the values used),
//   * which boards the loader accepts: patch:4606-4627 (tests/cpp/test_mapper.cpp check_unsupported),
//   * MMC3 registers -> PRG / CHR pages and mirroring: patch:4630-4681 (tests/cpp/test_reset_cart.cpp).
// Built and run by tests/test_oracle_kats.py; prints one line per failed check and exits non-zero on any.
#include <cstdio>
#include <exception>
#include <string>
#include <vector>

#include "nes.hpp"

namespace {

int g_failed = 0;

#define KAT(cond)                                                                  \
    do {                                                                           \
        if (!(cond)) {                                                             \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);            \
            ++g_failed;                                                            \
        }                                                                          \
    } while (0)

using namespace orc;

// ---------------------------------------------------------------------------------------------- DMC

constexpr u64 kByte = 8 * 54;   // rate 15: 54 CPU cycles per bit

struct DmcMachine {
    Cart cart;
    Console m{};
    u64 now = 1000;   // CPU cycles
    u64 stolen = 0;

    DmcMachine() {
        cart.prg.assign(32768, 0);
        cart.chr.assign(8192, 0);
        dmc_reset(m, now);
    }
    void write(u16 addr, u8 value) { cpu_write(cart, m, addr, value); }
    u8 status() { return cpu_read(cart, m, 0x4015); }
    // `cycles` worth of 4-cycle instructions, the DMC serviced after each one as the console step does
    void run(u64 cycles) {
        const u64 end = now + cycles;
        while (now < end) {
            now += 4;
            if (now >= m.dmc_event) {
                const u32 s = dmc_service(m, now, true);
                now += s;
                stolen += s;
            }
        }
    }
};

void dmc_kats() {
    {   // power-on is silent and an idle DMC never steals
        DmcMachine d;
        KAT(d.status() == 0x00);
        d.run(100 * kByte);
        KAT(d.stolen == 0);
        KAT(d.m.dmc_event == kDmcIdle);
    }
    {   // a 17-byte sample at rate 15: bit 4 until the last byte is fetched, 4 cycles per fetch
        DmcMachine d;
        d.run(3 * kByte + 100);
        d.write(0x4010, 0x0F);
        d.write(0x4013, 0x01);
        d.write(0x4015, 0x1F);
        KAT(d.status() == 0x10);
        d.run(4);   // the first byte is fetched after the starting instruction
        KAT(d.stolen == 4);
        d.run(15 * kByte - 2 * 4);
        KAT(d.status() == 0x10);
        d.run(2 * kByte);
        KAT(d.status() == 0x00);
        KAT(d.stolen == 17 * 4);
        d.run(10 * kByte);
        KAT(d.stolen == 17 * 4);
        d.write(0x4015, 0x10);   // bit 4 again restarts a finished sample
        KAT(d.status() == 0x10);
    }
    {   // bit 4 set while playing does not restart; bit 4 clear stops at once
        DmcMachine d;
        d.write(0x4010, 0x0F);
        d.write(0x4013, 0x01);
        d.write(0x4015, 0x10);
        d.run(4 * kByte);
        const u64 fetched = d.stolen / 4;
        KAT(fetched >= 4 && fetched <= 5);
        d.write(0x4015, 0x10);
        d.run(4 * kByte);
        KAT(d.stolen / 4 >= 8 && d.stolen / 4 <= 9);
        d.write(0x4015, 0x00);
        KAT(d.status() == 0x00);
        const u64 before = d.stolen;
        d.run(4 * kByte);
        KAT(d.stolen == before);
    }
    {   // loop flag: the sample restarts, bit 4 never clears, one fetch per byte
        DmcMachine d;
        d.write(0x4010, 0x4F);
        d.write(0x4013, 0x00);
        d.write(0x4015, 0x10);
        d.run(100 * kByte);
        KAT(d.status() == 0x10);
        KAT(d.stolen >= 100 * 4 && d.stolen <= 101 * 4);
    }
    {   // a rate change applies from the next bit clock: at rate 0 a byte lasts 8 x 428 cycles
        DmcMachine d;
        d.write(0x4010, 0x4F);
        d.write(0x4015, 0x10);
        d.run(10 * kByte);
        d.write(0x4010, 0x40);
        d.run(8 * 428);
        const u64 before = d.stolen;
        d.run(20 * 8 * 428);
        KAT(d.stolen - before >= 19 * 4 && d.stolen - before <= 21 * 4);
    }
    {   // fast-forwarded idle loop (no steal): bytes are consumed on time, the CPU loses no cycles
        DmcMachine d;
        d.write(0x4010, 0x0F);
        d.write(0x4013, 0x01);
        d.write(0x4015, 0x10);
        const u64 start = d.now;
        KAT(dmc_service(d.m, start, false) == 0);
        KAT(dmc_service(d.m, start + 10 * kByte, false) == 0);
        KAT(d.status() == 0x10);
        KAT(dmc_service(d.m, start + 17 * kByte, false) == 0);
        KAT(d.status() == 0x00);
    }
}

// ---------------------------------------------------------------------------------------------- replay renderer

struct RenderEnv {
    Cart cart;
    Console m{};
    std::vector<u8> frame = std::vector<u8>(256 * 240, 0);

    RenderEnv() {
        cart.prg.assign(32768, 0);
        cart.chr.assign(8192, 0);
        cart.board = kNrom;
        cart.arrangement = 0;   // vertical
        for (auto& b : m.oam) b = 0xFF;
    }
    // the live state as the frame to present (both banks from it, no writes), as the reference's frame_log_reset
    void reset_log() { log_reset(cart, m); }
    u32* shown() { return log_bank_ptr(m, m.log_bank & 1u); }
    // the whole 256 x 240 picture of the presented bank: the replay's colour numbers (render_obs without the crop)
    void draw() {
        const u32* h = shown();
        const Src src = make_src(cart, m, h, h[0] & ~kLogOverflow, m.snap_nt, m.snap_oam);
        RState s;
        r_load(s, h);
        RLine line;
        r_begin_frame(src, s);
        for (int l = 0; l < 240; ++l) {
            r_line(src, s, line, l, true);
            r_compose(s, line);
            for (int x = 0; x < 256; ++x) frame[l * 256 + x] = line.px[x] & 0x3F;
            r_end_of_line(src, s, l, true);
        }
    }
    bool pixel_is(int x, int y, u8 value) const { return frame[y * 256 + x] == value; }
};

void render_kats() {
    {   // background tile 1 at the top left, left column shown; then hidden
        RenderEnv e;
        e.cart.chr[0x0010] = 0x80;   // tile 1, row 0: leftmost pixel colour 1
        e.m.nt[0] = 0x01;
        e.m.pal[1] = 0x21;
        e.m.mask = 0x0A;
        e.reset_log();
        e.draw();
        KAT(e.pixel_is(0, 0, 0x21));
        KAT(e.pixel_is(1, 0, 0x00));
        KAT(e.pixel_is(0, 1, 0x00));
        KAT(e.pixel_is(8, 0, 0x00));
        e.m.mask = 0x08;
        e.reset_log();
        e.draw();
        KAT(e.pixel_is(0, 0, 0x00));
    }
    {   // a sprite at OAM y 9 is drawn from line 10, over a disabled background
        RenderEnv e;
        e.cart.chr[0x0020] = 0x80;   // tile 2, row 0: leftmost pixel colour 1
        e.m.pal[0x11] = 0x16;
        e.m.oam[0] = 9;
        e.m.oam[1] = 2;
        e.m.oam[2] = 0;
        e.m.oam[3] = 12;
        e.m.mask = 0x14;
        e.reset_log();
        e.draw();
        KAT(e.pixel_is(12, 10, 0x16));
        KAT(e.pixel_is(12, 9, 0x00));
        KAT(e.pixel_is(13, 10, 0x00));
    }
    {   // a logged $2005 write late on line 100 (after its fetches): the lines after it start 8 pixels to the right
        RenderEnv e;
        for (int row = 0; row < 8; ++row) e.cart.chr[0x0010 + row] = 0xFF;   // tile 1: every row colour 1
        for (int col = 0; col < 32; col += 2)
            for (int tile_row = 0; tile_row < 30; ++tile_row) e.m.nt[tile_row * 32 + col] = 0x01;
        e.m.pal[1] = 0x21;
        e.m.mask = 0x0A;
        e.reset_log();
        u32* h = e.shown();
        // $2005 = 8 (coarse x 1) by a 4-cycle store starting at NeSLE dot 100 * 341 + 240
        h[kLogHeader] = (100u * 341u + 240u) | (4u << 17) | (static_cast<u32>(kEvScroll) << 24);
        h[kLogHeader + 1] = 8u;
        h[0] = 1;
        e.draw();
        KAT(e.pixel_is(0, 50, 0x21) && e.pixel_is(8, 50, 0x00));
        KAT(e.pixel_is(0, 100, 0x21) && e.pixel_is(8, 100, 0x00));
        KAT(e.pixel_is(0, 101, 0x00) && e.pixel_is(8, 101, 0x21));
        KAT(e.pixel_is(0, 200, 0x00) && e.pixel_is(8, 200, 0x21));
    }
}

// ---------------------------------------------------------------------------------------------- boards

std::vector<u8> ines(u32 mapper, u32 prg, u32 chr) {
    std::vector<u8> r(16 + prg + chr, 0);
    r[0] = 'N'; r[1] = 'E'; r[2] = 'S'; r[3] = 0x1A;
    r[4] = static_cast<u8>(prg / 16384);
    r[5] = static_cast<u8>(chr / 8192);
    r[6] = static_cast<u8>((mapper & 0x0F) << 4);
    r[7] = static_cast<u8>(mapper & 0xF0);
    return r;
}

void board_kats() {
    for (u32 mapper : {1u, 3u, 4u, 9u}) {   // the paged boards, 64 KB PRG + 8 KB CHR
        const auto r = ines(mapper, 64 * 1024, 8 * 1024);
        bool ok = true;
        try { (void)parse_ines(r.data(), r.size()); } catch (const std::exception&) { ok = false; }
        KAT(ok);
    }
    for (u32 mapper : {7u, 66u, 71u, 255u}) {
        const auto r = ines(mapper, 64 * 1024, 8 * 1024);
        bool refused = false;
        try { (void)parse_ines(r.data(), r.size()); } catch (const std::exception& ex) {
            refused = std::string(ex.what()).find("unsupported mapper") != std::string::npos;
        }
        KAT(refused);
    }
    {   // MMC3 resumes from its registers: banks, mirroring (128 KB PRG, 128 KB CHR)
        Cart c;
        c.board = kMmc3;
        c.arrangement = 0;
        c.prg_page_mask = 15;
        c.chr_page_mask = 127;
        Console m{};
        const u8 level1[15] = {0, 0x3A, 0x4A, 0x5D, 0x6E, 0x61, 0x0A, 0x04, 0x46, 1, 0x80, 9, 7, 1, 0};
        for (int i = 0; i < 15; ++i) m.regs[i] = level1[i];
        board::sync(c, m);
        KAT(m.mirroring == kPageHorizontal);   // $A000 bit 0
        // bank select 0x46: PRG mode 1 puts R6 at $C000 and the second-last page at $8000
        KAT(m.prg_page[2] == (0x0Au << 13) && m.prg_page[0] == ((0x7Eu & 15u) << 13));
        KAT(m.prg_page[1] == (0x04u << 13) && m.prg_page[3] == (15u << 13));
        KAT(m.chr_page[4] == (0x4Au << 10) && m.chr_page[7] == (0x61u << 10));   // R2..R5, no CHR swap
        KAT(m.chr_page[2] == (0x3Au << 10) && m.chr_page[3] == (0x3Bu << 10));   // R1 as a 2 KB bank
    }
}

}  // namespace

int main() {
    dmc_kats();
    render_kats();
    board_kats();
    if (g_failed) {
        std::printf("%d known-answer checks failed\n", g_failed);
        return 1;
    }
    std::printf("all known-answer checks passed\n");
    return 0;
}
