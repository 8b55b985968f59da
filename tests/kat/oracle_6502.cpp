// TEST INFRASTRUCTURE: the oracle's 6502 core (oracle/nes.hpp Cpu::step) against the published behaviour of the
// NES's 2A03 (the MOS 6502 without decimal arithmetic). NeSLE's own core is not vendored, so these checks stand in
// for it: results, flags, cycle counts with their page-crossing and branch penalties, the stack, the JMP ($xxFF)
// page wrap, zero-page wraps, BRK / RTI, and unofficial opcodes faulting (the environment's definition).
// Built and run by tests/test_oracle_kats.py; prints one line per failed check and exits non-zero on any.
#include <cstdio>
#include <initializer_list>
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

struct Machine {
    Cart c;
    Console m{};
    Machine() {
        c.board = kNrom;
        c.prg.assign(32768, 0);
        c.chr.assign(8192, 0);
        c.prg[0x7FFE] = 0x00; c.prg[0x7FFF] = 0x90;   // BRK / IRQ vector: $9000
        m.sp = 0xFD;
        m.p = FU | FI;
    }
    // `code` at $0300 in RAM, run one instruction
    StepOut run(std::initializer_list<u8> code, u16 at = 0x0300) {
        u16 a = at;
        for (u8 b : code) m.ram[a++ & 0x7FF] = b;
        m.pc = at;
        Cpu cpu{c, m};
        return cpu.step();
    }
    bool flag(u8 f) const { return (m.p & f) != 0; }
};

void arithmetic() {
    Machine t;
    t.m.a = 0x50; t.m.p &= ~FC;
    CHECK(t.run({0x69, 0x50}).cycles == 2 && t.m.a == 0xA0 && t.flag(FV) && !t.flag(FC) && t.flag(FN));   // ADC #
    t.m.a = 0xFF; t.m.p &= ~FC;
    t.run({0x69, 0x01});
    CHECK(t.m.a == 0x00 && t.flag(FC) && t.flag(FZ) && !t.flag(FV));
    t.m.a = 0x09; t.m.p = static_cast<u8>((t.m.p | FD) & ~FC);      // decimal flag set: the 2A03 adds in binary
    t.run({0x69, 0x01});
    CHECK(t.m.a == 0x0A);
    t.m.a = 0x50; t.m.p |= FC;
    t.run({0xE9, 0xF0});                                             // SBC #
    CHECK(t.m.a == 0x60 && !t.flag(FC) && !t.flag(FV));
    t.m.a = 0x50; t.m.p |= FC;
    t.run({0xE9, 0xB0});
    CHECK(t.m.a == 0xA0 && !t.flag(FC) && t.flag(FV) && t.flag(FN));
    t.m.a = 0x40;
    t.run({0xC9, 0x40});                                             // CMP #
    CHECK(t.flag(FZ) && t.flag(FC) && !t.flag(FN));
    t.run({0xC9, 0x41});
    CHECK(!t.flag(FZ) && !t.flag(FC) && t.flag(FN));
    t.m.a = 0x80; t.m.p |= FC;
    t.run({0x2A});                                                   // ROL A: carry in, bit 7 out
    CHECK(t.m.a == 0x01 && t.flag(FC));
    t.m.ram[0x10] = 0xFF;
    CHECK(t.run({0xE6, 0x10}).cycles == 5 && t.m.ram[0x10] == 0x00 && t.flag(FZ));   // INC zp wraps
    t.m.a = 0xC0; t.m.ram[0x11] = 0x40;
    t.run({0x24, 0x11});                                             // BIT zp: N, V from memory, Z from A & M
    CHECK(!t.flag(FZ) && t.flag(FV) && !t.flag(FN));
}

void addressing_and_cycles() {
    Machine t;
    t.m.ram[0x0080] = 0x42;
    CHECK(t.run({0xA5, 0x80}).cycles == 3 && t.m.a == 0x42);                    // LDA zp
    t.m.x = 0x02; t.m.ram[0x0001] = 0x17;
    CHECK(t.run({0xB5, 0xFF}).cycles == 4 && t.m.a == 0x17);                    // LDA zp,X wraps in page zero
    t.m.x = 0x01; t.m.ram[0x0500] = 0x33;
    CHECK(t.run({0xBD, 0xFF, 0x04}).cycles == 5 && t.m.a == 0x33);             // LDA abs,X across a page: +1
    t.m.ram[0x04FF] = 0x34;
    CHECK(t.run({0xBD, 0xFE, 0x04}).cycles == 4 && t.m.a == 0x34);             // same page
    CHECK(t.run({0x9D, 0xFF, 0x04}).cycles == 5);                               // STA abs,X: 5 always
    t.m.ram[0x00FF] = 0x00; t.m.ram[0x0000] = 0x06; t.m.ram[0x0600] = 0x99; t.m.x = 0;
    CHECK(t.run({0xA1, 0xFF}).cycles == 6 && t.m.a == 0x99);                    // (zp,X): pointer wraps $FF -> $00
    t.m.ram[0x0020] = 0xF0; t.m.ram[0x0021] = 0x05; t.m.y = 0x20; t.m.ram[0x0610] = 0x77;
    CHECK(t.run({0xB1, 0x20}).cycles == 6 && t.m.a == 0x77);                    // (zp),Y across a page: +1
    CHECK(t.run({0x91, 0x20}).cycles == 6 && t.m.ram[0x0610] == 0x77);          // STA (zp),Y: 6 always
    t.m.x = 0x10;
    CHECK(t.run({0xFE, 0x00, 0x06}).cycles == 7 && t.m.ram[0x0610] == 0x78);    // INC abs,X: 7
}

void branches_and_jumps() {
    Machine t;
    t.m.p |= FZ;
    CHECK(t.run({0xD0, 0x10}).cycles == 2 && t.m.pc == 0x0302);                // BNE not taken
    CHECK(t.run({0xF0, 0x10}).cycles == 3 && t.m.pc == 0x0312);                // BEQ taken, same page
    CHECK(t.run({0xF0, 0x10}, 0x03F0).cycles == 4 && t.m.pc == 0x0402);        // taken into the next page
    CHECK(t.run({0xF0, 0xFC}, 0x0340).cycles == 3 && t.m.pc == 0x033E);        // backwards
    t.m.ram[0x02FF] = 0x34; t.m.ram[0x0200] = 0x12;
    CHECK(t.run({0x6C, 0xFF, 0x02}, 0x0400).cycles == 5 && t.m.pc == 0x1234);  // JMP ($02FF): high byte from $0200
    t.m.sp = 0xFD;
    CHECK(t.run({0x20, 0x00, 0x05}, 0x0310).cycles == 6 && t.m.pc == 0x0500);  // JSR pushes the address of its last byte
    CHECK(t.m.ram[0x01FD] == 0x03 && t.m.ram[0x01FC] == 0x12 && t.m.sp == 0xFB);
    CHECK(t.run({0x60}, 0x0500).cycles == 6 && t.m.pc == 0x0313 && t.m.sp == 0xFD);   // RTS: + 1
}

void stack_and_interrupts() {
    Machine t;
    t.m.p = FU | FC;
    CHECK(t.run({0x08}).cycles == 3 && t.m.ram[0x0100 | static_cast<u8>(t.m.sp + 1)] == (FU | FB | FC));   // PHP: B, U set
    t.m.ram[0x0100 | static_cast<u8>(t.m.sp + 1)] = 0xFF;
    CHECK(t.run({0x28}).cycles == 4 && t.m.p == static_cast<u8>(0xFF & ~FB));  // PLP: B not kept, U always set
    t.m.p = FU; t.m.sp = 0xFD;
    CHECK(t.run({0x00, 0xEA}, 0x0320).cycles == 7 && t.m.pc == 0x9000);         // BRK -> $FFFE vector
    CHECK(t.m.ram[0x01FD] == 0x03 && t.m.ram[0x01FC] == 0x22 && t.m.ram[0x01FB] == (FU | FB) && t.flag(FI));
    CHECK(t.run({0x40}, 0x0600).cycles == 6 && t.m.pc == 0x0322 && t.m.sp == 0xFD && !t.flag(FI));   // RTI
}

void unofficial_opcodes_fault() {
    Machine t;
    for (u8 op : {0x02, 0x1A, 0x80, 0xA7, 0xEB, 0xFF}) {
        const StepOut s = t.run({op, 0x00, 0x00});
        CHECK(s.illegal && s.opcode == op && s.pc == 0x0300);
    }
}

}  // namespace

int main() {
    arithmetic();
    addressing_and_cycles();
    branches_and_jumps();
    stack_and_interrupts();
    unofficial_opcodes_fault();
    if (g_failed) {
        std::printf("%d 6502 checks failed\n", g_failed);
        return 1;
    }
    std::printf("all 6502 checks passed\n");
    return 0;
}
