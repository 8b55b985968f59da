// MMC1 specialisation of the emulator, renderer and launch sequence (compiled as its own unit).
// Emulation blocks of 2 warps x 16 consoles sharing one PRG window: 3-6% less emulation time than 1 warp x 32
// on this board (MMC3, whose IRQ-split frames diverge more, is faster with 1 x 32 and keeps it).
#define GR_ENVS_PER_WARP 16
#define GR_FRAMES_WARPS 2
#include "host.cuh"

namespace gr {
GR_BOARD_TEMPLATES(, kMmc1)
}  // namespace gr
