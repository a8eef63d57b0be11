// Exposes the reference's tile encoder (cpu_bf16_reads.h pack_cpu_read_tiles,
// a FreeToken header vendored in edge35b) with a C ABI so the oracle's
// restatement can be checked against it.  The header is compiled where it
// lies in the reference tree (oracle/Makefile target `ref`); nothing of it is
// copied here.  Test infrastructure only.
#include <cstdint>
#include <cstddef>
#include "cpu_bf16_reads.h"

extern "C" size_t ref_pack_cpu_read_tiles(const uint16_t* raw, uint8_t* packed, uint8_t* bases,
                                          size_t tiles) {
    return freetoken::cpu_moe::pack_cpu_read_tiles(raw, packed, bases, tiles);
}
