"""Seeded synthetic NES cartridges and their reward10 specs.

Commercial ROMs are not available, so every workload runs on cartridges built here from a seed: a fixed 6502
program template (assembled by the small two-pass assembler below) with seed-derived constants, uniform random CHR
tiles and a uniform random nametable. The template is the one the benchmark configs describe:

  reset:  PPU off, two vblank waits, RAM cleared, palette + both nametables uploaded, OAM buffer with 8 seed-placed
          sprites, lives/LFSR/mode set, NMI + rendering on, then ``JMP *`` (the idle loop the emulator fast-forwards)
  NMI:    OAM DMA from $0200 ($4014); scroll from the progress word; controller read ($4016) into zp $00;
          progress $10-11 += velocity while Right is held (-= while Left, clamped at 0); level $12 += 1 when the
          progress high byte reaches the threshold; a 16-bit Galois LFSR (the pad byte XORed into its low byte
          every frame) decides hazards: one low-byte value and clear high bits decrement lives $13 (game over,
          mode $17 = 2, at 0), one high-byte value knocks progress back; A adds a BCD digit to the 3-byte score
          $14-16; the player sprite follows progress.

Board variants (mapper 2 UxROM, 1 MMC1, 4 MMC3) add the bank traffic the configs name: UxROM switches its 16 KB
window on every level change, MMC1 rewrites its PRG bank through the serial port every 64 frames and uploads its
CHR into CHR-RAM at reset, MMC3 arms its scanline IRQ for line 32 each frame and its IRQ handler writes a new scroll
(a mid-frame split the renderer must replay). CNROM switches its 8 KB CHR bank on every level change. MMC2 (mapper 9)
draws from both 4 KB halves through its $FD/$FE latches: the random nametable and two sprites carry $FD/$FE tiles
that flip them mid-line, the NMI puts $0FD8/$0FE8 and $1FD8/$1FE8 on the PPU bus ($2006 + a $2007 read) by frame
parity, every 64th frame it waits into the picture and rewrites a CHR register and $2006 there (logged mid-frame
register and latch changes), and every level change switches the $8000 PRG page.

The reward side is a 13th reward10 reader (`SYNTH_READER`): RAM $10-$17 -> Signals, with per-game seeded fp32
weights promoted to float64 (`reward_spec`).
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

# ----------------------------------------------------------------------------------------------- 6502 assembler

# (mnemonic, mode) -> opcode, official NMOS 6502 instructions only.
_OPS = {}
_ROWS = {
    'ADC': dict(imm=0x69, zp=0x65, zpx=0x75, abs=0x6D, absx=0x7D, absy=0x79, indx=0x61, indy=0x71),
    'AND': dict(imm=0x29, zp=0x25, zpx=0x35, abs=0x2D, absx=0x3D, absy=0x39, indx=0x21, indy=0x31),
    'ASL': dict(acc=0x0A, zp=0x06, zpx=0x16, abs=0x0E, absx=0x1E),
    'BIT': dict(zp=0x24, abs=0x2C),
    'CMP': dict(imm=0xC9, zp=0xC5, zpx=0xD5, abs=0xCD, absx=0xDD, absy=0xD9, indx=0xC1, indy=0xD1),
    'CPX': dict(imm=0xE0, zp=0xE4, abs=0xEC),
    'CPY': dict(imm=0xC0, zp=0xC4, abs=0xCC),
    'DEC': dict(zp=0xC6, zpx=0xD6, abs=0xCE, absx=0xDE),
    'EOR': dict(imm=0x49, zp=0x45, zpx=0x55, abs=0x4D, absx=0x5D, absy=0x59, indx=0x41, indy=0x51),
    'INC': dict(zp=0xE6, zpx=0xF6, abs=0xEE, absx=0xFE),
    'JMP': dict(abs=0x4C, ind=0x6C),
    'JSR': dict(abs=0x20),
    'LDA': dict(imm=0xA9, zp=0xA5, zpx=0xB5, abs=0xAD, absx=0xBD, absy=0xB9, indx=0xA1, indy=0xB1),
    'LDX': dict(imm=0xA2, zp=0xA6, zpy=0xB6, abs=0xAE, absy=0xBE),
    'LDY': dict(imm=0xA0, zp=0xA4, zpx=0xB4, abs=0xAC, absx=0xBC),
    'LSR': dict(acc=0x4A, zp=0x46, zpx=0x56, abs=0x4E, absx=0x5E),
    'ORA': dict(imm=0x09, zp=0x05, zpx=0x15, abs=0x0D, absx=0x1D, absy=0x19, indx=0x01, indy=0x11),
    'ROL': dict(acc=0x2A, zp=0x26, zpx=0x36, abs=0x2E, absx=0x3E),
    'ROR': dict(acc=0x6A, zp=0x66, zpx=0x76, abs=0x6E, absx=0x7E),
    'SBC': dict(imm=0xE9, zp=0xE5, zpx=0xF5, abs=0xED, absx=0xFD, absy=0xF9, indx=0xE1, indy=0xF1),
    'STA': dict(zp=0x85, zpx=0x95, abs=0x8D, absx=0x9D, absy=0x99, indx=0x81, indy=0x91),
    'STX': dict(zp=0x86, zpy=0x96, abs=0x8E),
    'STY': dict(zp=0x84, zpx=0x94, abs=0x8C),
}
for _m, _modes in _ROWS.items():
    for _mode, _op in _modes.items():
        _OPS[(_m, _mode)] = _op
_IMPLIED = dict(BRK=0x00, CLC=0x18, CLD=0xD8, CLI=0x58, CLV=0xB8, DEX=0xCA, DEY=0x88, INX=0xE8, INY=0xC8,
                NOP=0xEA, PHA=0x48, PHP=0x08, PLA=0x68, PLP=0x28, RTI=0x40, RTS=0x60, SEC=0x38, SED=0xF8,
                SEI=0x78, TAX=0xAA, TAY=0xA8, TSX=0xBA, TXA=0x8A, TXS=0x9A, TYA=0x98)
_BRANCH = dict(BCC=0x90, BCS=0xB0, BEQ=0xF0, BMI=0x30, BNE=0xD0, BPL=0x10, BVC=0x50, BVS=0x70)
_SIZE = dict(imp=1, acc=1, imm=2, zp=2, zpx=2, zpy=2, indx=2, indy=2, rel=2, abs=3, absx=3, absy=3, ind=3)


def opcode_table():
    """(mnemonic, mode) -> opcode for every official instruction (used by tests as an independent decode table)."""
    t = dict(_OPS)
    t.update({(m, 'imp'): o for m, o in _IMPLIED.items()})
    t.update({(m, 'rel'): o for m, o in _BRANCH.items()})
    return t


class Asm:
    """Two-pass assembler: emit instructions with symbolic operands, then `assemble()` resolves the labels.

    `a.i('LDA', 'imm', 3)`, `a.i('STA', 'abs', 0x2000)`, `a.i('BNE', 'rel', 'loop')`, `a.i('INX')`;
    operands may be ints, label names, or ('<' | '>', label) for a label's low / high byte.
    """

    def __init__(self, org: int):
        self.org = org
        self.items = []       # (addr, kind, payload)
        self.labels = {}
        self.pc = org

    def label(self, name):
        assert name not in self.labels, name
        self.labels[name] = self.pc

    def i(self, mnem, mode=None, arg=None):
        if mode is None:
            mode = 'rel' if mnem in _BRANCH else 'imp'
        if mode == 'rel':
            op = _BRANCH[mnem]
        elif mode == 'imp':
            op = _IMPLIED[mnem]
        else:
            op = _OPS[(mnem, mode)]
        self.items.append((self.pc, 'op', (op, mode, arg)))
        self.pc += _SIZE[mode]

    def bytes(self, data):
        data = bytes(data)
        self.items.append((self.pc, 'raw', data))
        self.pc += len(data)

    def word(self, arg):
        self.items.append((self.pc, 'word', arg))
        self.pc += 2

    def _val(self, arg):
        if isinstance(arg, tuple):
            part, name = arg
            v = self.labels[name]
            return v & 0xFF if part == '<' else v >> 8
        if isinstance(arg, str):
            return self.labels[arg]
        return int(arg)

    def assemble(self) -> dict:
        """addr -> byte for every emitted byte."""
        out = {}
        for addr, kind, payload in self.items:
            if kind == 'raw':
                for k, b in enumerate(payload):
                    out[addr + k] = b
            elif kind == 'word':
                v = self._val(payload)
                out[addr], out[addr + 1] = v & 0xFF, (v >> 8) & 0xFF
            else:
                op, mode, arg = payload
                out[addr] = op
                if mode in ('imp', 'acc'):
                    continue
                v = self._val(arg)
                if mode == 'rel':
                    d = v - (addr + 2)
                    assert -128 <= d <= 127, f'branch out of range at {addr:04x}'
                    out[addr + 1] = d & 0xFF
                elif _SIZE[mode] == 2:
                    assert 0 <= v <= 0xFF, (mode, v)
                    out[addr + 1] = v
                else:
                    out[addr + 1], out[addr + 2] = v & 0xFF, (v >> 8) & 0xFF
        return out


# ------------------------------------------------------------------------------------------------- cartridges

MAPPERS = {'nrom': 0, 'mmc1': 1, 'uxrom': 2, 'cnrom': 3, 'mmc3': 4, 'mmc2': 9}

# zero page / RAM map of the template (the synthetic reward reader reads these)
ZP_BUTTONS, ZP_TMP, ZP_LFSR, ZP_FRAME = 0x00, 0x01, 0x02, 0x04
ZP_PTR = 0x06
ZP_DMC = 0x08   # the DMC variant keeps each frame's $4015 read here
ZP_COUNT = 0x0A   # loop counter of the mid-frame PPU variants
ZP_PROGRESS, ZP_LEVEL, ZP_LIVES, ZP_SCORE, ZP_MODE = 0x10, 0x12, 0x13, 0x14, 0x17
OAM_BUF = 0x0200


@dataclasses.dataclass
class Cart:
    board: str
    seed: int
    rom: bytes            # iNES image
    boot_pads: bytes      # pad byte of every boot frame (power-on -> first controllable frame)
    params: dict          # the seed-derived template constants


def _template(a: Asm, p: dict, board: str, data_labels: dict, dmc: bool = False, ppu: str | None = None):
    """The reset/NMI/IRQ program (see the module docstring); `dmc`: the NMI also plays a DMC sample; `ppu`: the NMI
    ends with one of the mid-frame PPU programs of `_ppu_variant`."""
    i = a.i
    # ---------------------------------------------------------------- reset
    a.label('reset')
    i('SEI'); i('CLD'); i('LDX', 'imm', 0xFF); i('TXS')
    i('LDA', 'imm', 0); i('STA', 'abs', 0x2000); i('STA', 'abs', 0x2001)
    a.label('vw1'); i('BIT', 'abs', 0x2002); i('BPL', 'rel', 'vw1')
    i('LDA', 'imm', 0); i('TAX')
    a.label('clr')
    for page in range(8):
        i('STA', 'absx', page * 0x100)
    i('INX'); i('BNE', 'rel', 'clr')
    a.label('vw2'); i('BIT', 'abs', 0x2002); i('BPL', 'rel', 'vw2')
    if board == 'mmc1':
        # control: 8 KB CHR mode off (4 KB), PRG mode 3, vertical mirroring = %01110 -> serial write
        _mmc1_write(a, 0x8000, 0x0E, 'c')
        _mmc1_write(a, 0xE000, 0x00, 'p')
        # CHR-RAM upload: 8 KB from CHRTAB through $2007
        i('LDA', 'imm', 0x00); i('STA', 'abs', 0x2006); i('STA', 'abs', 0x2006)
        i('LDA', 'imm', ('<', 'chrtab')); i('STA', 'zp', ZP_PTR)
        i('LDA', 'imm', ('>', 'chrtab')); i('STA', 'zp', ZP_PTR + 1)
        i('LDX', 'imm', 32); i('LDY', 'imm', 0)
        a.label('chr'); i('LDA', 'indy', ZP_PTR); i('STA', 'abs', 0x2007); i('INY'); i('BNE', 'rel', 'chr')
        i('INC', 'zp', ZP_PTR + 1); i('DEX'); i('BNE', 'rel', 'chr')
    if board == 'mmc2':
        # PRG page 0 at $8000; CHR registers $B000 / $C000 (the $0000 half's $FD / $FE banks), $D000 / $E000 (the
        # $1000 half's); vertical mirroring
        for reg, v in zip((0xA000, 0xB000, 0xC000, 0xD000, 0xE000, 0xF000), [0] + list(p['creg']) + [0]):
            i('LDA', 'imm', v); i('STA', 'abs', reg)
    if board == 'mmc3':
        # PRG mode 0, CHR mode 0; R0..R5 = 0, 2, 4, 5, 6, 7 (the first 8 KB of CHR), vertical mirroring
        for r, v in enumerate([0, 2, 4, 5, 6, 7]):
            i('LDA', 'imm', r); i('STA', 'abs', 0x8000); i('LDA', 'imm', v); i('STA', 'abs', 0x8001)
        i('LDA', 'imm', 0); i('STA', 'abs', 0xA000)
    # palette
    i('LDA', 'imm', 0x3F); i('STA', 'abs', 0x2006); i('LDA', 'imm', 0x00); i('STA', 'abs', 0x2006)
    i('LDX', 'imm', 0)
    a.label('pal'); i('LDA', 'absx', 'paltab'); i('STA', 'abs', 0x2007); i('INX'); i('CPX', 'imm', 32)
    i('BNE', 'rel', 'pal')
    # both nametables (2 KB)
    i('LDA', 'imm', 0x20); i('STA', 'abs', 0x2006); i('LDA', 'imm', 0x00); i('STA', 'abs', 0x2006)
    i('LDA', 'imm', ('<', 'nttab')); i('STA', 'zp', ZP_PTR)
    i('LDA', 'imm', ('>', 'nttab')); i('STA', 'zp', ZP_PTR + 1)
    i('LDX', 'imm', 8); i('LDY', 'imm', 0)
    a.label('nt'); i('LDA', 'indy', ZP_PTR); i('STA', 'abs', 0x2007); i('INY'); i('BNE', 'rel', 'nt')
    i('INC', 'zp', ZP_PTR + 1); i('DEX'); i('BNE', 'rel', 'nt')
    # OAM buffer: every sprite hidden, then the 8 placed ones
    i('LDA', 'imm', 0xFF); i('LDX', 'imm', 0)
    a.label('hide'); i('STA', 'absx', OAM_BUF); i('INX'); i('BNE', 'rel', 'hide')
    i('LDX', 'imm', 0)
    a.label('spr'); i('LDA', 'absx', 'sprtab'); i('STA', 'absx', OAM_BUF); i('INX'); i('CPX', 'imm', 32)
    i('BNE', 'rel', 'spr')
    # game state
    i('LDA', 'imm', p['lives']); i('STA', 'zp', ZP_LIVES)
    i('LDA', 'imm', p['lfsr'] & 0xFF); i('STA', 'zp', ZP_LFSR)
    i('LDA', 'imm', p['lfsr'] >> 8); i('STA', 'zp', ZP_LFSR + 1)
    i('LDA', 'imm', 1); i('STA', 'zp', ZP_MODE)
    a.label('vw3'); i('BIT', 'abs', 0x2002); i('BPL', 'rel', 'vw3')
    i('LDA', 'imm', 0); i('STA', 'abs', 0x2005); i('STA', 'abs', 0x2005)
    i('LDA', 'imm', p['ctrl']); i('STA', 'abs', 0x2000)
    i('LDA', 'imm', p['mask']); i('STA', 'abs', 0x2001)
    if board == 'mmc3':
        i('CLI')
    a.label('main'); i('JMP', 'abs', 'main')

    # ---------------------------------------------------------------- NMI
    a.label('nmi')
    i('PHA'); i('TXA'); i('PHA'); i('TYA'); i('PHA')
    i('LDA', 'imm', 0); i('STA', 'abs', 0x2003); i('LDA', 'imm', OAM_BUF >> 8); i('STA', 'abs', 0x4014)
    i('BIT', 'abs', 0x2002)
    if dmc:
        # a 17-byte sample at rate 15, looped on odd frames, (re)started by $4015 bit 4 each frame; the status byte
        # goes to RAM. Its fetches steal CPU cycles from the instructions that run while it plays.
        i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 1)
        for _ in range(6):
            i('ASL', 'acc')
        i('ORA', 'imm', 0x0F); i('STA', 'abs', 0x4010)
        i('LDA', 'imm', 0x01); i('STA', 'abs', 0x4013)
        i('LDA', 'imm', 0x1F); i('STA', 'abs', 0x4015)
        i('LDA', 'abs', 0x4015); i('STA', 'zp', ZP_DMC)
    if board == 'mmc2':
        # latch 0 <- $FD / $FE by frame bit 0, latch 1 by frame bit 1: $2006 puts the address on the bus, a $2007 read
        # puts it there again (and its successor)
        for half, bit in ((0x0F, 0), (0x1F, 1)):
            i('LDA', 'imm', half); i('STA', 'abs', 0x2006)
            i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 1 << bit)
            for _ in range(4 - bit):
                i('ASL', 'acc')
            i('CLC'); i('ADC', 'imm', 0xD8); i('STA', 'abs', 0x2006)
            i('LDA', 'abs', 0x2007)
    if board == 'mmc3':
        # top of the frame unscrolled; the IRQ at line 32 sets the playfield scroll
        i('LDA', 'imm', 0); i('STA', 'abs', 0x2005); i('STA', 'abs', 0x2005)
        i('LDA', 'imm', p['ctrl']); i('STA', 'abs', 0x2000)
        i('LDA', 'imm', p['irq_line'] - 1); i('STA', 'abs', 0xC000); i('STA', 'abs', 0xC001)
        i('STA', 'abs', 0xE001)
    else:
        i('LDA', 'zp', ZP_PROGRESS); i('STA', 'abs', 0x2005); i('LDA', 'imm', 0); i('STA', 'abs', 0x2005)
        i('LDA', 'zp', ZP_PROGRESS + 1); i('AND', 'imm', 1); i('ORA', 'imm', p['ctrl']); i('STA', 'abs', 0x2000)
    # controller -> zp $00 (bit 7 A ... bit 0 Right)
    i('LDA', 'imm', 1); i('STA', 'abs', 0x4016); i('LDA', 'imm', 0); i('STA', 'abs', 0x4016)
    i('LDX', 'imm', 8)
    a.label('rd'); i('LDA', 'abs', 0x4016); i('LSR', 'acc'); i('ROL', 'zp', ZP_BUTTONS); i('DEX')
    i('BNE', 'rel', 'rd')
    i('LDA', 'zp', ZP_MODE); i('CMP', 'imm', 1); i('BEQ', 'rel', 'play'); i('JMP', 'abs', 'nmi_out')
    a.label('play')
    i('INC', 'zp', ZP_FRAME); i('BNE', 'rel', 'fr_ok'); i('INC', 'zp', ZP_FRAME + 1)
    a.label('fr_ok')
    if board == 'mmc1':
        # every 64 frames: PRG bank = (frame / 64) & 7 through the serial port
        i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 0x3F); i('BNE', 'rel', 'nobank')
        i('LDA', 'zp', ZP_FRAME); i('LSR', 'acc'); i('LSR', 'acc'); i('LSR', 'acc'); i('LSR', 'acc')
        i('LSR', 'acc'); i('LSR', 'acc'); i('STA', 'zp', ZP_TMP)
        i('LDA', 'zp', ZP_FRAME + 1); i('ASL', 'acc'); i('ASL', 'acc'); i('ORA', 'zp', ZP_TMP)
        i('AND', 'imm', 0x07)
        for _ in range(5):
            i('STA', 'abs', 0xE000); i('LSR', 'acc')
        i('LDA', 'abs', 0x8000); i('STA', 'abs', OAM_BUF + 9)   # the new bank's first byte becomes a tile
        a.label('nobank')
    # Right / Left move the progress word
    i('LDA', 'zp', ZP_BUTTONS); i('AND', 'imm', 0x01); i('BEQ', 'rel', 'noright')
    i('CLC'); i('LDA', 'zp', ZP_PROGRESS); i('ADC', 'imm', p['vel']); i('STA', 'zp', ZP_PROGRESS)
    i('LDA', 'zp', ZP_PROGRESS + 1); i('ADC', 'imm', 0); i('STA', 'zp', ZP_PROGRESS + 1)
    a.label('noright')
    i('LDA', 'zp', ZP_BUTTONS); i('AND', 'imm', 0x02); i('BEQ', 'rel', 'noleft')
    i('SEC'); i('LDA', 'zp', ZP_PROGRESS); i('SBC', 'imm', p['vel']); i('TAX')
    i('LDA', 'zp', ZP_PROGRESS + 1); i('SBC', 'imm', 0); i('BCC', 'rel', 'clamp0')
    i('STA', 'zp', ZP_PROGRESS + 1); i('STX', 'zp', ZP_PROGRESS); i('JMP', 'abs', 'noleft')
    a.label('clamp0'); i('LDA', 'imm', 0); i('STA', 'zp', ZP_PROGRESS); i('STA', 'zp', ZP_PROGRESS + 1)
    a.label('noleft')
    # level: progress high byte reaches the threshold
    i('LDA', 'zp', ZP_PROGRESS + 1); i('CMP', 'imm', p['thresh']); i('BCC', 'rel', 'nolevel')
    i('SBC', 'imm', p['thresh']); i('STA', 'zp', ZP_PROGRESS + 1); i('INC', 'zp', ZP_LEVEL)
    if board == 'cnrom':   # CHR bank = level & 3 (written over an equal ROM byte, as a bus-conflict-safe game would)
        i('LDA', 'zp', ZP_LEVEL); i('AND', 'imm', 0x03); i('TAX')
        i('LDA', 'absx', 'banktab'); i('STA', 'absx', 'banktab')
    if board == 'mmc2':
        i('LDA', 'zp', ZP_LEVEL); i('AND', 'imm', 0x0F); i('STA', 'abs', 0xA000)
        i('LDA', 'abs', 0x8000); i('STA', 'abs', OAM_BUF + 9)
    if board == 'uxrom':
        i('LDA', 'zp', ZP_LEVEL); i('AND', 'imm', 0x07); i('TAX')
        i('LDA', 'absx', 'banktab'); i('STA', 'absx', 'banktab')
        i('LDA', 'abs', 0x8000); i('STA', 'abs', OAM_BUF + 9)
    a.label('nolevel')
    # A: score += digit (BCD, 3 bytes)
    i('LDA', 'zp', ZP_BUTTONS); i('AND', 'imm', 0x80); i('BEQ', 'rel', 'noscore')
    i('JSR', 'abs', 'bcd_add')
    a.label('noscore')
    # LFSR step (16-bit Galois, taps $B400), then the pad byte mixed in (trajectories depend on the actions)
    i('LSR', 'zp', ZP_LFSR + 1); i('ROR', 'zp', ZP_LFSR); i('BCC', 'rel', 'nox')
    i('LDA', 'zp', ZP_LFSR + 1); i('EOR', 'imm', 0xB4); i('STA', 'zp', ZP_LFSR + 1)
    a.label('nox')
    i('LDA', 'zp', ZP_LFSR); i('EOR', 'zp', ZP_BUTTONS); i('STA', 'zp', ZP_LFSR)
    # hazard: a life lost
    i('LDA', 'zp', ZP_LFSR); i('CMP', 'imm', p['haz_lo']); i('BNE', 'rel', 'nohaz')
    i('LDA', 'zp', ZP_LFSR + 1); i('AND', 'imm', p['haz_hi']); i('BNE', 'rel', 'nohaz')
    i('DEC', 'zp', ZP_LIVES); i('BNE', 'rel', 'nohaz')
    i('LDA', 'imm', 2); i('STA', 'zp', ZP_MODE)
    a.label('nohaz')
    # knock-back: progress high byte -= knock (clamped at 0)
    i('LDA', 'zp', ZP_LFSR + 1); i('AND', 'imm', p['kn_mask']); i('CMP', 'imm', p['kn_val']); i('BNE', 'rel', 'nokn')
    i('LDA', 'zp', ZP_PROGRESS + 1); i('SEC'); i('SBC', 'imm', p['kn_hi']); i('BCS', 'rel', 'knok')
    i('LDA', 'imm', 0); i('STA', 'zp', ZP_PROGRESS)
    a.label('knok'); i('STA', 'zp', ZP_PROGRESS + 1)
    a.label('nokn')
    # player sprite (sprite 1) follows progress
    i('LDA', 'zp', ZP_PROGRESS); i('LSR', 'acc'); i('STA', 'abs', OAM_BUF + 7)
    a.label('nmi_out')
    if ppu is not None:
        _ppu_variant(a, p, ppu)
    if board == 'mmc2':
        # every 64th frame: wait ~2,400 cycles in 7-cycle instructions (into the picture, about line 10), then
        # rewrite the $FE bank of the $0000 half and put $1FD8 on the bus (the rest of the frame is drawn from there)
        i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 0x3F); i('BNE', 'rel', 'nosplit')
        i('LDX', 'imm', 0); i('LDY', 'imm', 40)
        a.label('dly')
        for _ in range(8):
            i('ROL', 'absx', 0x0700)
        i('DEY'); i('BNE', 'rel', 'dly')
        i('LDA', 'zp', ZP_LEVEL); i('AND', 'imm', 0x0F); i('ORA', 'imm', 0x10); i('STA', 'abs', 0xC000)
        i('LDA', 'imm', 0x1F); i('STA', 'abs', 0x2006); i('LDA', 'imm', 0xD8); i('STA', 'abs', 0x2006)
        a.label('nosplit')
    i('PLA'); i('TAY'); i('PLA'); i('TAX'); i('PLA')
    i('RTI')

    # ---------------------------------------------------------------- IRQ (MMC3 split)
    a.label('irq')
    if board == 'mmc3':
        i('PHA')
        i('STA', 'abs', 0xE000)
        i('LDA', 'zp', ZP_PROGRESS); i('STA', 'abs', 0x2005); i('LDA', 'imm', 0); i('STA', 'abs', 0x2005)
        i('LDA', 'zp', ZP_PROGRESS + 1); i('AND', 'imm', 1); i('ORA', 'imm', p['ctrl']); i('STA', 'abs', 0x2000)
        i('PLA')
    i('RTI')

    # ---------------------------------------------------------------- BCD add of one digit into $14-$16
    a.label('bcd_add')
    i('LDX', 'imm', 2); i('LDA', 'imm', p['score_add']); i('STA', 'zp', ZP_TMP)
    a.label('bcd_loop')
    i('LDA', 'zpx', ZP_SCORE); i('AND', 'imm', 0x0F); i('CLC'); i('ADC', 'zp', ZP_TMP); i('CMP', 'imm', 0x0A)
    i('BCC', 'rel', 'bcd_lo'); i('ADC', 'imm', 0x05)
    a.label('bcd_lo'); i('STA', 'zp', ZP_TMP)
    i('LDA', 'zpx', ZP_SCORE); i('AND', 'imm', 0xF0); i('CLC'); i('ADC', 'zp', ZP_TMP); i('CMP', 'imm', 0xA0)
    i('BCC', 'rel', 'bcd_store'); i('SBC', 'imm', 0xA0); i('STA', 'zpx', ZP_SCORE)
    i('LDA', 'imm', 1); i('STA', 'zp', ZP_TMP); i('DEX'); i('BPL', 'rel', 'bcd_loop'); i('RTS')
    a.label('bcd_store'); i('STA', 'zpx', ZP_SCORE); i('RTS')

    # ---------------------------------------------------------------- data
    for name, data in data_labels.items():
        a.label(name)
        a.bytes(data)


PPU_VARIANTS = ('split', 'raster', 'vread')


def _delay(a: Asm, tag: str, outer: int, inner: int):
    """About outer * (inner * 5 + 4) CPU cycles: nested DEX / DEY loops."""
    a.i('LDY', 'imm', outer)
    a.label(tag + '_o'); a.i('LDX', 'imm', inner & 0xFF)
    a.label(tag + '_i'); a.i('DEX'); a.i('BNE', 'rel', tag + '_i')
    a.i('DEY'); a.i('BNE', 'rel', tag + '_o')


def _ppu_variant(a: Asm, p: dict, kind: str):
    """Mid-frame PPU programs run at the end of the NMI, the ways real games drive the PPU while it draws:

    split   SMB-style status bar: wait for the sprite-0 flag of the last frame to clear (pre-render line), poll
            $2002 bit 6 until sprite 0 hits (bounded: ~25,000 cycles, then give up for this frame), then, in the
            middle of that line, a $2006 pair (moves the VRAM address at once) and a $2005 pair (the scroll the next
            line's horizontal copy takes).
    raster  wait into the picture, then 6 times: rendering off, one palette entry rewritten through $2006 / $2007,
            the VRAM address put back into the nametable, rendering (background + sprites) on again, a few lines
            apart: more palette versions in one frame than the walk keeps, lines drawn with rendering off, and
            rendering switched back on inside lines or their hblank.
    vread   wait into the picture, then 3 $2007 reads a few lines apart with rendering on (the read buffer refill
            moves the VRAM address as the PPU's own increments do).
    """
    i = a.i
    assert kind in PPU_VARIANTS, kind
    if kind == 'split':
        a.label('s0_clear'); i('BIT', 'abs', 0x2002); i('BVS', 'rel', 's0_clear')
        i('LDY', 'imm', 9)
        a.label('s0_o'); i('LDX', 'imm', 0)
        a.label('s0_i'); i('BIT', 'abs', 0x2002); i('BVS', 'rel', 's0_hit'); i('DEX'); i('BNE', 'rel', 's0_i')
        i('DEY'); i('BNE', 'rel', 's0_o'); i('JMP', 'abs', 's0_end')
        a.label('s0_hit')
        i('LDA', 'imm', 0x21); i('STA', 'abs', 0x2006); i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 0xE0)
        i('STA', 'abs', 0x2006)
        i('LDA', 'zp', ZP_PROGRESS); i('STA', 'abs', 0x2005); i('LDA', 'zp', ZP_FRAME); i('AND', 'imm', 0x0F)
        i('STA', 'abs', 0x2005)
        a.label('s0_end')
        return
    _delay(a, kind + '_in', 3, 0)   # ~3,900 cycles: from the NMI's end past the pre-render line into the picture
    if kind == 'raster':
        i('LDA', 'imm', 6); i('STA', 'zp', ZP_COUNT)
        a.label('ras')
        i('LDX', 'imm', 120); a.label('ras_d'); i('DEX'); i('BNE', 'rel', 'ras_d')   # ~600 cycles, ~5 lines
        i('LDA', 'imm', 0x00); i('STA', 'abs', 0x2001)
        i('LDA', 'imm', 0x3F); i('STA', 'abs', 0x2006)
        i('LDA', 'zp', ZP_COUNT); i('ASL', 'acc'); i('ASL', 'acc'); i('ASL', 'acc'); i('ORA', 'imm', 0x01)
        i('AND', 'imm', 0x1F); i('STA', 'abs', 0x2006)
        i('LDA', 'zp', ZP_FRAME); i('EOR', 'zp', ZP_COUNT); i('AND', 'imm', 0x3F); i('STA', 'abs', 0x2007)
        i('LDA', 'imm', 0x20); i('STA', 'abs', 0x2006); i('LDA', 'zp', ZP_COUNT); i('STA', 'abs', 0x2006)
        i('LDA', 'imm', p['mask']); i('STA', 'abs', 0x2001)
        i('DEC', 'zp', ZP_COUNT); i('BNE', 'rel', 'ras')
        return
    i('LDA', 'imm', 3); i('STA', 'zp', ZP_COUNT)
    a.label('vr')
    i('LDX', 'zp', ZP_LFSR); a.label('vr_d'); i('DEX'); i('BNE', 'rel', 'vr_d')   # 5..1,280 cycles, by the LFSR
    i('LDA', 'abs', 0x2007)
    i('DEC', 'zp', ZP_COUNT); i('BNE', 'rel', 'vr')


def _mmc1_write(a: Asm, addr: int, value: int, tag: str):
    """Serial MMC1 register write of a constant (reset bit first)."""
    a.i('LDA', 'imm', 0x80); a.i('STA', 'abs', 0x8000)
    a.i('LDA', 'imm', value)
    for _ in range(5):
        a.i('STA', 'abs', addr); a.i('LSR', 'acc')


def template_params(seed: int, board: str) -> dict:
    r = np.random.default_rng([seed, 0x5EED])
    haz_bits = int(r.integers(1, 4))           # one life lost per ~2^(8 + bits) frames
    ctrl = 0x80 | (0x08 if board == 'mmc3' else int(r.choice([0x08, 0x10])) if board == 'mmc2'
                   else int(r.choice([0x00, 0x08, 0x10, 0x18])))
    emph = int(r.choice([0, 0, 0, 1, 2, 4]))
    p = dict(
        vel=int(r.integers(1, 7)),
        thresh=int(r.integers(4, 13)),
        lives=int(r.integers(2, 6)),
        lfsr=int(r.integers(1, 0x10000)),
        haz_lo=int(r.integers(1, 256)), haz_hi=(1 << haz_bits) - 1,
        kn_mask=0xFF, kn_val=int(r.integers(0, 256)),
        kn_hi=int(r.integers(1, 4)),
        score_add=int(r.integers(1, 10)),
        ctrl=ctrl,
        mask=0x1E | (emph << 5),
        irq_line=32,
    )
    if board == 'mmc2':   # the four CHR registers ($FD/$FE banks of each half): distinct 4 KB banks of 32
        p['creg'] = [int(b) for b in r.permutation(32)[:4]]
    return p


def make_cart(seed: int, board: str = 'nrom', dmc: bool = False, ppu: str | None = None) -> Cart:
    """A seeded synthetic cartridge (iNES image + boot pads); `dmc`: a variant whose NMI plays a DMC sample every
    frame (the registered games never do; tests use it for the sample channel and its cycle steals); `ppu`: a variant
    whose NMI ends with a mid-frame PPU program (`PPU_VARIANTS`, see `_ppu_variant`; not on MMC2, whose NMI has its own
    mid-frame writes), for the sequential renderer and the CPU-visible sprite-0 flag."""
    assert board in MAPPERS, board
    assert ppu is None or board != 'mmc2', 'the MMC2 cart has its own mid-frame program'

    p = template_params(seed, board)
    r = np.random.default_rng([seed, 0xC0DE])
    chr_bytes = r.integers(0, 256, 8192, dtype=np.uint8).tobytes()
    nt = r.integers(0, 256, 2048, dtype=np.uint8).tobytes()
    pal = r.integers(0, 64, 32, dtype=np.uint8).tobytes()
    spr = bytearray()
    for k in range(8):
        y = int(r.integers(0, 224)) if k != 1 else 150
        tile = int(r.integers(0, 256))
        if board == 'mmc2' and k in (3, 4):
            tile = 0xFD if k == 3 else 0xFE   # sprite fetches that flip a latch on their lines
        spr += bytes([y, tile, int(r.integers(0, 256)) & 0xE3, int(r.integers(0, 248))])
    prg_size = {'nrom': 32768, 'cnrom': 32768, 'uxrom': 131072, 'mmc1': 131072, 'mmc3': 262144, 'mmc2': 131072}[board]
    data = dict(paltab=pal, nttab=nt, sprtab=bytes(spr))
    if board == 'uxrom':
        data['banktab'] = bytes(range(8))
    if board == 'cnrom':
        data['banktab'] = bytes(range(4))
    if board == 'mmc1':
        data['chrtab'] = chr_bytes
    # program in the last 16 KB (fixed bank on every board), vectors at $FFFA
    a = Asm(0xC000)
    _template(a, p, board, data, dmc, ppu)
    img = a.assemble()
    assert max(img) < 0xFFFA, 'program overflows into the vectors'
    prg = bytearray(r.integers(0, 256, prg_size, dtype=np.uint8).tobytes())
    base = prg_size - 0x4000
    for addr, b in img.items():
        prg[base + addr - 0xC000] = b
    vec = struct.pack('<HHH', a.labels['nmi'], a.labels['reset'], a.labels['irq'])
    prg[prg_size - 6:] = vec
    mapper = MAPPERS[board]
    chr_rom = b'' if board == 'mmc1' else chr_bytes   # MMC1: CHR-RAM, filled by the reset code from CHRTAB
    if board == 'mmc3':
        r.integers(0, 256, 131072, dtype=np.uint8)   # skipped: the cart's bytes stay those every earlier build drew
        chr_rom = bytes(chr_bytes) + r.integers(0, 256, 131072 - 8192, dtype=np.uint8).tobytes()
    if board == 'cnrom':   # 4 CHR banks of 8 KB
        chr_rom = bytes(chr_bytes) + r.integers(0, 256, 32768 - 8192, dtype=np.uint8).tobytes()
    if board == 'mmc2':    # 32 banks of 4 KB
        chr_rom = bytes(chr_bytes) + r.integers(0, 256, 131072 - 8192, dtype=np.uint8).tobytes()
    flags6 = ((mapper & 0x0F) << 4) | 0x01          # vertical mirroring
    flags7 = mapper & 0xF0
    header = b'NES\x1a' + bytes([prg_size // 16384, len(chr_rom) // 8192, flags6, flags7]) + bytes(8)
    rom = header + bytes(prg) + chr_rom
    boot = bytes(12 if board != 'mmc1' else 16)   # power-on to the first frame with NMI on and rendering
    return Cart(board=board, seed=seed, rom=rom, boot_pads=boot, params=p)


# ----------------------------------------------------------------------------------------------- reward specs

# Layout of the per-game reward parameters handed to the native libraries (float64 each), in this order.
SPEC_FIELDS = ('progress_unit', 'score_unit', 'stall_frames', 'idle_per_frame', 'death_from_lives', 'start_ok',
               'select_ok', 'w_progress', 'w_level', 'w_death', 'w_damage', 'w_score', 'score_cap',
               'score_level_budget', 'w_win', 'w_stall', 'w_rollback', 'rollback_drop', 'reader', 'frame_limit')
READER_SYNTH = 1.0   # 'reader' field value of the synthetic RAM reader ($10-$17 of the template)
FIRST_SYNTH_GAME = 12   # rl10 game ids 0..11 are the reference's commercial games


def reward_spec(seed: int, cart_params: dict | None = None) -> np.ndarray:
    """Seeded reward10 parameters of one synthetic game id: fp32 weights promoted to float64 (exact), the
    reference's structure (progress, level, death, capped score, stall, rollback; no damage or win term)."""
    r = np.random.default_rng([seed, 0x4E3A])
    f32 = lambda lo, hi: float(np.float32(r.uniform(lo, hi)))  # noqa: E731
    thresh = (cart_params or {}).get('thresh', 8)
    stall_s = float(int(r.integers(8, 31)))
    w = dict(
        progress_unit=float(thresh * 256), score_unit=float(int(r.integers(5, 50)) * 10),
        stall_frames=stall_s * 60.0, idle_per_frame=0.0, death_from_lives=1.0, start_ok=0.0, select_ok=0.0,
        w_progress=f32(0.5, 1.5), w_level=f32(0.5, 1.5), w_death=-f32(0.05, 0.3), w_damage=0.0,
        w_score=f32(0.005, 0.05), score_cap=f32(0.05, 0.2), score_level_budget=f32(0.1, 0.4), w_win=0.0,
        w_stall=-f32(0.05, 0.3), w_rollback=-f32(0.01, 0.05), rollback_drop=0.25, reader=READER_SYNTH,
        frame_limit=18000.0)
    w_idle = -f32(1.0, 2.5)
    w['idle_per_frame'] = w_idle / (stall_s * 60.0)
    return np.array([w[k] for k in SPEC_FIELDS], dtype=np.float64)
