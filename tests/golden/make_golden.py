"""Generate golden fixtures by running the reference's own Python modules.

Run in a container where the reference checkout is available (its path is the
first argument, default ``../reference`` relative to the repo root's parent is
NOT assumed; pass it explicitly):

    python tests/golden/make_golden.py /path/to/reference

The reference needs ``diffusers`` only for class names in its import lines;
a stub module stands in for it.  The LTX RoPE table class needs the full
diffusers ``ModelMixin`` machinery at import time, so its class body is taken
from ``models/dits/eraserdit_transformer.py`` with ``ast`` and executed alone.
diffusers ``RMSNorm`` (diffusers==0.40.0, absent here) is restated from its
published ``forward`` as ``DiffusersRMSNorm`` below: fp32 mean of squares,
``x * rsqrt(var + eps)``, rounded to the 16-bit weight dtype, times the weight.
The reference's own Triton "native" kernel documents the same rounding
boundaries (``layers/operator_fusion/triton/rmsnorm_native.py:1-5,25-43``).
``torch.nn.RMSNorm`` of torch 2.11 rounds once instead of twice and is NOT used.

Fixtures are small: selected token rows plus whole-tensor checksums.  The test
regenerates the seeded inputs with ``eraserdit_b200.synthetic`` and compares.
"""

from __future__ import annotations

import ast
import importlib.abc
import importlib.machinery
import json
import math
import sys
import types
from pathlib import Path
from types import SimpleNamespace
from unittest.mock import patch

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from eraserdit_b200.synthetic import CONFIG0, make_hidden, make_params  # noqa: E402

ROWS = list(range(0, 192, 24)) + [191]


def install_diffusers_stub() -> None:
    import torch.nn as nn

    class _Dummy(nn.Module):
        def __init__(self, *args, **kwargs):
            super().__init__()

    class _Stub(types.ModuleType):
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            if name in ("register_to_config", "maybe_allow_in_graph"):
                return lambda f: f
            if name == "logging":
                import logging
                return SimpleNamespace(get_logger=logging.getLogger)
            if name == "USE_PEFT_BACKEND":
                return False
            return type(name, (_Dummy,), {})

    class _Finder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
        def find_spec(self, fullname, path, target=None):
            if fullname == "diffusers" or fullname.startswith("diffusers."):
                return importlib.machinery.ModuleSpec(fullname, self, is_package=True)
            return None

        def create_module(self, spec):
            return _Stub(spec.name)

        def exec_module(self, module):
            module.__path__ = []

    sys.meta_path.insert(0, _Finder())


class DiffusersRMSNorm(torch.nn.Module):
    """diffusers 0.40.0 ``models.normalization.RMSNorm`` (affine, no bias)."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(dim))

    def forward(self, hidden_states):
        variance = hidden_states.to(torch.float32).pow(2).mean(-1, keepdim=True)
        hidden_states = hidden_states * torch.rsqrt(variance + self.eps)
        if self.weight.dtype in (torch.float16, torch.bfloat16):
            hidden_states = hidden_states.to(self.weight.dtype)
        return hidden_states * self.weight


def load_reference_rope_class(reference: Path):
    source = (reference / "models/dits/eraserdit_transformer.py").read_text()
    tree = ast.parse(source)
    node = next(n for n in tree.body
                if isinstance(n, ast.ClassDef) and n.name == "LTXVideoRotaryPosEmbed")
    module = ast.Module(body=[node], type_ignores=[])
    from typing import Optional, Tuple
    namespace = dict(torch=torch, nn=torch.nn, math=math, Optional=Optional, Tuple=Tuple)
    exec(compile(module, "eraserdit_transformer.py", "exec"), namespace)
    return namespace["LTXVideoRotaryPosEmbed"]


def rows(t: torch.Tensor) -> np.ndarray:
    return t[:, ROWS].detach().float().numpy()


def checksums(t: torch.Tensor) -> dict:
    t = t.detach().double()
    return dict(sum=t.sum().item(), sumsq=t.square().sum().item(),
                channel_sum=t.sum(dim=(0, 1)).numpy(), token_sumsq=t.square().sum(-1).numpy())


def main(reference: Path) -> None:
    install_diffusers_stub()
    sys.path.insert(0, str(reference))
    from models.dits.eraserdit_attention import EraserDiTAttentionProcessor, apply_rotary_emb
    from models.adapters.eraserdit.nccl_sequence import DistributedSequenceRank
    from parallel.sequence_sharding import plan_sequence_shards
    from config.dit_parallel import DiTTopology
    import models.dits.eraserdit_attention as attention_module

    out: dict[str, np.ndarray] = {}
    rope_cls = load_reference_rope_class(reference)
    rope = rope_cls(dim=2048, base_num_frames=20, base_height=2048, base_width=2048,
                    patch_size=1, patch_size_t=1, theta=10000.0)
    cfg = CONFIG0
    hs = torch.zeros(cfg.batch, cfg.seq, 2048)
    cos, sin = rope(hs, cfg.frames, cfg.height, cfg.width, rope_interpolation_scale=None)
    out["rope_int_cos_rows"], out["rope_int_sin_rows"] = rows(cos), rows(sin)
    out["rope_int_cos_sum"] = np.array(cos.double().sum().item())
    out["rope_int_sin_sum"] = np.array(sin.double().sum().item())
    scale = (8.0 / 25.0, 32.0, 32.0)
    cos_s, sin_s = rope(hs, cfg.frames, cfg.height, cfg.width, rope_interpolation_scale=scale)
    out["rope_scaled_cos_rows"], out["rope_scaled_sin_rows"] = rows(cos_s), rows(sin_s)

    # ---- one full self-attention layer through the reference processor (fp32 CPU)
    params = make_params(cfg.seed, cfg.eps)
    x = make_hidden(cfg)

    def build_attn(p, dtype):
        attn = torch.nn.Module()
        attn.heads = 32
        attn.to_q = torch.nn.Linear(2048, 2048)
        attn.to_k = torch.nn.Linear(2048, 2048)
        attn.to_v = torch.nn.Linear(2048, 2048)
        attn.to_out = torch.nn.ModuleList([torch.nn.Linear(2048, 2048), torch.nn.Dropout(0.0)])
        attn.norm_q = DiffusersRMSNorm(2048, eps=p.eps)
        attn.norm_k = DiffusersRMSNorm(2048, eps=p.eps)
        with torch.no_grad():
            for lin, w, b in ((attn.to_q, p.wq, p.bq), (attn.to_k, p.wk, p.bk),
                              (attn.to_v, p.wv, p.bv), (attn.to_out[0], p.wo, p.bo)):
                lin.weight.copy_(w)
                lin.bias.copy_(b)
            attn.norm_q.weight.copy_(p.norm_q)
            attn.norm_k.weight.copy_(p.norm_k)
        return attn.to(dtype).eval()

    captured = {}
    processor = EraserDiTAttentionProcessor(attention_backend="sdpa")
    original_resolve = processor._resolve_self_attention

    def resolve(query, *, has_attn_mask):
        selection, impl = original_resolve(query, has_attn_mask=has_attn_mask)
        forward = impl.forward

        class Capture:
            causal = impl.causal
            softmax_scale = impl.softmax_scale

            def forward(self, q, k, v, m):
                result = forward(q, k, v, m)
                captured["core"] = result
                return result
        return selection, Capture()

    processor._resolve_self_attention = resolve
    with torch.no_grad():
        attn = build_attn(params, torch.float32)
        layer = processor(attn, x, image_rotary_emb=(cos, sin))
    out["layer0_fp32_rows"] = rows(layer)
    for key, value in checksums(layer).items():
        out[f"layer0_fp32_{key}"] = np.asarray(value)
    out["core0_fp32_rows"] = rows(captured["core"].flatten(2, 3))
    for key, value in checksums(captured["core"].flatten(2, 3)).items():
        out[f"core0_fp32_{key}"] = np.asarray(value)

    # bf16 run of the same layer through the reference (CPU bf16 arithmetic)
    with torch.no_grad():
        attn16 = build_attn(params, torch.bfloat16)
        layer16 = processor(attn16, x.bfloat16(), image_rotary_emb=(cos, sin))
    out["layer0_bf16_rows"] = rows(layer16)

    # ---- QK RMSNorm + RoPE in bf16 (the fusion op's reference closure)
    g = torch.Generator().manual_seed(72)
    for tag, shape, amp, eps in (("a", (1, 9, 2048), 100.0, 1e-5),
                                 ("b", (2, 5, 2048), 0.001, 1e-6)):
        q = (torch.randn(shape, generator=g) * amp).bfloat16()
        k = (torch.randn(shape, generator=g) * amp).bfloat16()
        wq = (torch.rand(2048, generator=g) * 4 - 2).bfloat16()
        wk = (torch.rand(2048, generator=g) * 1.6 + 0.2).bfloat16()
        angles = torch.randn(shape, generator=g)
        qn = DiffusersRMSNorm(2048, eps=eps).bfloat16()
        kn = DiffusersRMSNorm(2048, eps=eps).bfloat16()
        with torch.no_grad():
            qn.weight.copy_(wq)
            kn.weight.copy_(wk)
            freqs = (angles.cos(), angles.sin())
            rq = apply_rotary_emb(qn(q), freqs)
            rk = apply_rotary_emb(kn(k), freqs)
        out[f"qk_{tag}_q"] = q.view(torch.int16).numpy()
        out[f"qk_{tag}_k"] = k.view(torch.int16).numpy()
        out[f"qk_{tag}_wq"] = wq.view(torch.int16).numpy()
        out[f"qk_{tag}_wk"] = wk.view(torch.int16).numpy()
        out[f"qk_{tag}_angles"] = angles.numpy()
        out[f"qk_{tag}_eps"] = np.array(eps)
        out[f"qk_{tag}_out_q"] = rq.view(torch.int16).numpy()
        out[f"qk_{tag}_out_k"] = rk.view(torch.int16).numpy()

    # ---- Ulysses wire layout (reference packing with a fake collective)
    wires = {}
    for degree, length, batch in ((2, 16, 1), (4, 19, 3)):
        heads, dim = 8, 4
        full = torch.arange(batch * length * heads * dim, dtype=torch.float32).reshape(
            batch, length, heads, dim)
        for rank in range(degree):
            groups = SimpleNamespace(topology=SimpleNamespace(sp=degree, ulysses=degree),
                                     coordinates=(0, rank, 0),
                                     get=lambda name, r=rank, d=degree: (None, tuple(range(d)), r))
            with patch.dict("os.environ", MGERASE_NCCL_PACKING="packed"):
                seq = DistributedSequenceRank(groups)
            local = full[:, seq.partition(length)]
            seen = {}

            def collective(output, packed, output_splits, input_splits, group):
                seen["wire"] = packed.clone()
                seen["splits"] = (list(output_splits), list(input_splits))
                output.zero_()
            with patch("models.adapters.eraserdit.nccl_sequence.dist.all_to_all_single",
                       collective):
                seq._ulysses_input(local)
            key = f"wire_in_d{degree}_l{length}_b{batch}_r{rank}"
            out[key] = seen["wire"].numpy()
            wires[key] = seen["splits"]

    # ---- host logic: shard plans and CFG x SP topologies
    host = {"ulysses_splits": wires, "plans": {}, "topology": {}}
    for length, degree in ((32640, 2), (32640, 4), (32640, 8), (19, 4), (7, 8), (0, 3)):
        plans = plan_sequence_shards(length, degree, 0)
        host["plans"][f"{length}_{degree}"] = [
            [p.global_length, p.padded_length, p.local_start, p.local_end,
             p.valid_local_length, p.pad_right] for p in plans]
    for name, topo in (("sp8", DiTTopology(ulysses=8)), ("cfg2_sp4", DiTTopology(ulysses=4, cfg=2)),
                       ("cfg2_sp2", DiTTopology(ulysses=2, cfg=2))):
        host["topology"][name] = {
            axis: [list(r) for r in topo.groups(axis)] for axis in ("ulysses", "sp", "cfg")}
        host["topology"][name]["coordinates"] = [list(topo.coordinates(r))
                                                 for r in range(topo.world_size)]
    lengths = {}
    for length, degree in ((32640, 8), (19, 4), (7, 3)):
        lengths[f"{length}_{degree}"] = [
            length * (r + 1) // degree - length * r // degree for r in range(degree)]
    host["floor_lengths"] = lengths

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    (HERE / "reference_host.json").write_text(json.dumps(host, indent=1, sort_keys=True))
    print("wrote", HERE / "reference_golden.npz", "and reference_host.json")
    del attention_module


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    main(Path(sys.argv[1]))
