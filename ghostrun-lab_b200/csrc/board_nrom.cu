// NROM specialisation of the emulator, renderer and launch sequence (compiled as its own unit).
// Emulation blocks of 2 warps x 16 consoles sharing one PRG window: 6% less emulation time than 1 warp x 32 when
// the board runs alone (config 2). The other boards keep 1 x 32: with several games' kernels running at once
// (config 3) the 2 x 16 shape on every board lost 5%.
#define GR_ENVS_PER_WARP 16
#define GR_FRAMES_WARPS 2
#include "host.cuh"

namespace gr {
GR_BOARD_TEMPLATES(, kNrom)
}  // namespace gr
