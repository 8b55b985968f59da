"""The reference's known-answer tests for its emulator extensions (DMC channel and $4015, frame-log replay renderer;
third_party/nesle-extensions.patch:4065-4207, 4355-4522), restated in tests/kat/oracle_kat.cpp against the CPU
oracle's own functions, compiled here with g++ and run. This pins those parts of the oracle to the reference's
expected values; the GPU parity tests then hold the product bit-exact to the oracle."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_passes_the_reference_known_answer_tests(tmp_path):
    exe = tmp_path / 'oracle_kat'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_kat.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all known-answer checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_mmc2_follows_the_reference_board(tmp_path):
    """MMC2 in the oracle against the patch's board code (registers, pages, latch hook ranges and their order
    around the $2007 buffer, frame-log events, the replay's fetch hook): tests/kat/oracle_mmc2.cpp."""
    exe = tmp_path / 'oracle_mmc2'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_mmc2.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all MMC2 checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_paged_boards_follow_the_reference(tmp_path):
    """MMC1's serial port and modes, CNROM's latch, MMC3's revision-B counter and its clock timing in the oracle
    against the patch's board code: tests/kat/oracle_boards.cpp."""
    exe = tmp_path / 'oracle_boards'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_boards.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all board checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_frame_log_follows_the_reference(tmp_path):
    """The frame log in the oracle against the patch's recording code (event encoding, the $2007 merge with rendering
    off, vblank, overflow, cycle stamps, FCEUmm's time base, the emphasis tint): tests/kat/oracle_framelog.cpp."""
    exe = tmp_path / 'oracle_framelog'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_framelog.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all frame-log checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_ppu_timing_follows_the_reference(tmp_path):
    """The PPU's timing events (vblank flag, NMI, status clear, log freeze / capture, sprite-0 scheduling) and the
    sprite-0 hit dot in the oracle against the patch's step code: tests/kat/oracle_ppu.cpp."""
    exe = tmp_path / 'oracle_ppu'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_ppu.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all PPU timing checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_6502_follows_the_published_2a03(tmp_path):
    """The oracle's 6502 core against the NES 2A03's published behaviour (binary-only ADC / SBC, flags, cycle counts
    and penalties, stack, JMP ($xxFF), zero-page wraps, BRK / RTI, unofficial opcodes faulting): NeSLE's core is not
    vendored, so this stands in for it. tests/kat/oracle_6502.cpp."""
    exe = tmp_path / 'oracle_6502'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_6502.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all 6502 checks passed' in run.stdout


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_oracle_bus_follows_the_published_nes(tmp_path):
    """The oracle's CPU bus against the NES's published register behaviour ($2002, the $2005 / $2006 toggle, the
    $2007 read buffer and palette reads, v steps, palette mirrors, the controller port, OAM DMA timing, nametable
    mirroring): NeSLE's base bus is not vendored, so this stands in for it. tests/kat/oracle_bus.cpp."""
    exe = tmp_path / 'oracle_bus'
    build = subprocess.run(['g++', '-std=c++17', '-O1', '-ffp-contract=off', '-I', str(ROOT / 'oracle'),
                            str(ROOT / 'tests' / 'kat' / 'oracle_bus.cpp'), '-o', str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-1000:]
    assert 'all bus checks passed' in run.stdout
