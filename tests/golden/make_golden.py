"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree is checked out (REFERENCE_ROOT, default a
sibling directory `reference` next to this repository) after
`make -C oracle ref`:

    python tests/golden/make_golden.py

Layer fixtures (layer_*.npz) come from the installed transformers
Qwen3_5MoeSparseMoeBlock -- the eager expert body edge35b pins by AST hash
(edge35b/expert_stream.py:28-33) -- run on CPU with the synthetic weights of
lightreason_b200.synthetic.  The router adds the benchmark configs' per-expert
bias to the FP32 logits before the softmax (the one deviation from
modeling_qwen3_5_moe.py:762-770) and casts the renormalised scores to BF16, the
dtype the reference's fast paths require (edge35b/fused_experts.py:41-42).

Codec fixtures (codec_vectors.npz) come from edge35b/bf16_expert_codec.py and
from edge35b/gpu_resident_experts.encode with FreeToken's pack_cpu_read_tiles
supplied by the reference's own cpu_bf16_reads.h (oracle/_ref/libref_tiles.so),
on the input vectors of the reference's tests
(test_freetoken_packed_transfer.py:15-26, :127-149; test_gpu_resident_experts.py:13-23).
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from lightreason_b200 import synthetic as S  # noqa: E402

LAYER_CASES = [  # (tokens, seed, bias kind)
    (1, 11, "normal"),
    (8, 12, "normal"),
    (16, 13, "normal"),
    (64, 14, "zipf"),
]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def t_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def make_layer(tokens: int, seed: int, bias_kind: str) -> None:
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock

    torch.manual_seed(0)
    config = Qwen3_5MoeTextConfig(hidden_size=2048, moe_intermediate_size=512, num_experts=256,
                                  num_experts_per_tok=8, shared_expert_intermediate_size=512)
    config._experts_implementation = "eager"
    with torch.device("meta"):
        block = Qwen3_5MoeSparseMoeBlock(config)
    block = block.to_empty(device="cpu").to(torch.bfloat16).eval().requires_grad_(False)
    w = S.layer_weights(seed, bias=bias_kind)
    gu, dn = w.stacked()
    with torch.no_grad():
        block.gate.weight.copy_(t_bf16(w.router))
        block.experts.gate_up_proj.copy_(t_bf16(gu))
        block.experts.down_proj.copy_(t_bf16(dn))
        block.shared_expert.gate_proj.weight.copy_(t_bf16(w.sh_gate))
        block.shared_expert.up_proj.weight.copy_(t_bf16(w.sh_up))
        block.shared_expert.down_proj.weight.copy_(t_bf16(w.sh_down))
        block.shared_expert_gate.weight.copy_(t_bf16(w.sh_gate_w).reshape(1, -1))
    x_bits = S.hidden_states(seed, tokens)
    x = t_bf16(x_bits)
    bias = torch.from_numpy(w.bias)
    F = torch.nn.functional
    with torch.no_grad():
        shared = block.shared_expert(x)                                   # TF:709
        logits = F.linear(x, block.gate.weight)                           # TF:764
        probs = F.softmax(logits.float() + bias, dim=-1)                  # TF:765 (+ bias)
        top_v, top_i = torch.topk(probs, 8, dim=-1)                       # TF:766
        top_v = top_v / top_v.sum(dim=-1, keepdim=True)                   # TF:767
        scores = top_v.to(torch.bfloat16)
        routed = block.experts(x, top_i, scores)                          # TF:727-751 eager
        out = routed + F.sigmoid(block.shared_expert_gate(x)) * shared    # TF:788-790
    z = logits.float() + bias
    zs = torch.sort(z, dim=-1, descending=True).values
    path = HERE / f"layer_T{tokens}_s{seed}.npz"
    np.savez_compressed(
        path, tokens=tokens, seed=seed, bias_kind=bias_kind,
        idx=top_i.numpy(), scores=scores.view(torch.int16).numpy().view(np.uint16),
        scores_f32=top_v.float().numpy(), logits=logits.view(torch.int16).numpy().view(np.uint16),
        out=out.view(torch.int16).numpy().view(np.uint16),
        margin_k=(zs[:, 7] - zs[:, 8]).numpy(),
        weights_sha256=digest(w.router, w.bias, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w, gu, dn),
        routed_sha256=digest(*[a for e in sorted(set(top_i.reshape(-1).tolist())) for a in (gu[e], dn[e])]),
        x_sha256=digest(x_bits),
        transformers_version=__import__("transformers").__version__)
    print(f"wrote {path.name}: out max {out.abs().max().item():.4f}")


def _reference_modules():
    root = Path(os.environ.get("REFERENCE_ROOT", str(ROOT.parent / "reference")))
    sys.path.insert(0, str(root))
    so = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_tiles.so"))
    so.ref_pack_cpu_read_tiles.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_size_t]
    so.ref_pack_cpu_read_tiles.restype = ctypes.c_size_t
    # FreeToken is not vendored; its pack_cpu_read_tiles is the reference's
    # cpu_bf16_reads.h compiled by oracle/Makefile.
    ft, kern, cpu = (types.ModuleType(n) for n in ("freetoken", "freetoken.kernel", "freetoken.kernel._cpu_moe"))
    cpu.pack_cpu_read_tiles = lambda src, packed, bases, n: so.ref_pack_cpu_read_tiles(src, packed, bases, n)
    ft.kernel, kern._cpu_moe = kern, cpu
    sys.modules.update({"freetoken": ft, "freetoken.kernel": kern, "freetoken.kernel._cpu_moe": cpu})
    import edge35b.bf16_expert_codec as codec
    import edge35b.gpu_resident_experts as resident
    return codec, resident, so


def make_codec() -> None:
    codec, resident, tiles = _reference_modules()
    out = {}
    # test_freetoken_packed_transfer.py:15-26: every BF16 bit pattern.
    values = np.arange(65536, dtype=np.uint16)
    base, escapes = codec.exponent_window(values)
    packed = np.empty(codec.row_bytes(values.size, escapes), dtype=np.uint8)
    codec.pack_verified_row(values, packed, base, escapes)
    out.update(all_base=base, all_escapes=escapes, all_packed_sha256=digest(packed))
    common = np.full(values.shape, 0x3F80, dtype=np.uint16)
    plans, size = codec.plan_bank(np.stack([common, values, common]))
    out.update(plan_none=np.array([p is None for p in plans]), plan_size=size,
               plan_rows=np.array([p if p is not None else (-1, -1, -1) for p in plans], dtype=np.int64))
    # test_freetoken_packed_transfer.py:127-149: mixed raw/packed bank, seed 76.
    rng = np.random.default_rng(76)
    for n in (64, 32):
        bits = rng.integers(0, 2 ** 16, (4, n), dtype=np.uint16)
        bits[2:] = (bits[2:] & 0x807F) | ((120 + (bits[2:] & 7)) << 7)
        bits[2, [0, 7, n - 1]] = [0x8000, 0x7F81, 0xFFFF]
        out[f"mixed{n}_bits"] = bits
        for expert in (2, 3):
            b, e = codec.exponent_window(bits[expert])
            row = np.empty(codec.row_bytes(n, e), dtype=np.uint8)
            codec.pack_verified_row(bits[expert], row, b, e)
            out[f"mixed{n}_e{expert}_packed"] = row
            out[f"mixed{n}_e{expert}_meta"] = np.array([b, e], dtype=np.int64)
    # test_gpu_resident_experts.py:13-23: 24 encoded + 8 raw tiles, seed 7091.
    gen = torch.Generator().manual_seed(7091)
    words = torch.randint(0, 128, (32, 256), generator=gen, dtype=torch.int32)
    words |= torch.randint(0, 2, words.shape, generator=gen, dtype=torch.int32) << 15
    exponents = 118 + torch.randint(0, 8, words.shape, generator=gen, dtype=torch.int32)
    exponents[1::4] = torch.arange(256) % 128
    words |= exponents << 7
    original = words.to(torch.int16).view(torch.bfloat16)
    data, headers, encoded, fallback = resident.encode(original)
    out.update(tiles7091_bits=original.view(torch.int16).numpy().view(np.uint16), tiles7091_data=data,
               tiles7091_headers=headers, tiles7091_counts=np.array([encoded, fallback]))
    # The tile encoder itself (non-compact layout) on the same words.
    raw = np.ascontiguousarray(original.view(torch.int16).numpy().view(np.uint16))
    tp = np.zeros(32 * 384, dtype=np.uint8)
    tb = np.zeros(32, dtype=np.uint8)
    n_enc = tiles.ref_pack_cpu_read_tiles(raw.ctypes.data, tp.ctypes.data, tb.ctypes.data, 32)
    out.update(tiles7091_packed=tp, tiles7091_bases=tb, tiles7091_encoded=n_enc)
    path = HERE / "codec_vectors.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path.name}: all-pattern base {base} escapes {escapes}; 7091 tiles {encoded}+{fallback}")


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    make_codec()
    for case in LAYER_CASES:
        make_layer(*case)
