"""Drop-in for edge35b/native_bf16_gather.py on B200.

Same geometry tuples, names and `copy` signature as the reference's
NativeBf16Gather (edge35b/native_bf16_gather.py:7-77): descriptor tables,
destinations, sizes, source/destination ids and a device-side count, launched
on the torch current stream, so a copy can be captured in a CUDA graph and
replayed with a different count.  The kernels are the sm_100a ones of
libmoe_b200.so (moe_gather_rows) instead of NVRTC-compiled Ada code, so there
is no capability-8.9 check; the constructor requires an sm_100 device.
"""

from __future__ import annotations

import torch

from lightreason_b200 import native

NATIVE_GEOMETRIES = (
    (4, 256, "default"), (8, 128, "default"), (8, 256, "default"), (16, 128, "default"),
    (8, 256, "l2"), (16, 128, "l2"),
)
CPU_TILE_GEOMETRIES = ((4, 256, "cpu-tiles"), (8, 128, "cpu-tiles"), (16, 128, "cpu-tiles"))

_CODECS = {"default": native.CODEC_ROW, "l2": native.CODEC_ROW_L2, "cpu-tiles": native.CODEC_TILES,
           "resident": native.CODEC_RESIDENT}


def name(geometry) -> str:
    return "cuda-" + "-".join(map(str, geometry))


def select_geometry(tag: str, *, shared: bool = False):
    for geometry in CPU_TILE_GEOMETRIES if shared else NATIVE_GEOMETRIES:
        if name(geometry) == tag:
            return geometry
    raise ValueError(f"Unknown B200 gather geometry {tag!r}.")


class NativeBf16Gather:
    """Descriptor-driven BF16 expert copies into cache slots (see module doc)."""

    def __init__(self):
        if not torch.cuda.is_available():
            raise RuntimeError("The B200 gather needs a CUDA device.")
        torch.cuda.init()
        native.device_check(torch.cuda.current_device())
        self.functions = dict(_CODECS)

    def copy(self, descriptors, destinations, sizes, src, dst, count, *, max_copies, experts, geometry):
        stripes, threads, policy = geometry
        if policy not in self.functions:
            raise ValueError(f"Unknown gather policy {policy!r}")
        native.gather_rows(descriptors, destinations, sizes, src, dst, count, max_copies=max_copies,
                           experts=experts, codec=self.functions[policy], stripes=stripes, threads=threads)

    def stage_primary(self, sources, miss_sources, layouts, prefix_tables, plan, count, *, experts, packed_slots):
        """edge35b/native_bf16_gather.py:79-84: stage the plan's experts as BF16
        rows (packed-slot hit, or miss from the source / replica with a slot
        refill); plan int32 [3, rows] (expert, slot, miss), count int32 [1]."""
        native.stage_primary(sources, miss_sources, layouts, prefix_tables, plan, count, experts=experts,
                             packed_slots=packed_slots)

    def copy_compact_tail(self, sources, destinations, sizes, prefixes, tail, src, dst, count, entries, resident,
                          experts):
        """edge35b/native_bf16_gather.py:86-93: BF16 rows into their slots; a
        cacheable miss also writes its compact bytes into its tail entry."""
        native.gather_compact_tail(sources, destinations, sizes, prefixes, tail, src, dst, count, entries, resident,
                                   experts=experts)
