// CNROM specialisation of the emulator, renderer and launch sequence (compiled as its own unit).
#include "host.cuh"

namespace gr {
GR_BOARD_TEMPLATES(, kCnrom)
}  // namespace gr
