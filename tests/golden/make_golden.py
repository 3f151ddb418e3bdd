"""Generate the golden fixtures from the REFERENCE's own legacy Pairformer block.

Run in the build container only (it imports the FoldForge source tree, which does not
travel to GPU boxes): ``python tests/golden/make_golden.py --reference <FoldForge checkout>/src``.

For every case it

1. draws the block's engine-key weights with :func:`foldforge_b200.synthetic.block_state`,
2. maps them to the RELEASED layout (the inverse of ``legacy/released.py:135-369``),
   loads them strictly into the reference's ``legacy.pairformer.PairformerBlock`` and
   checks that the reference's own converter ``pairformer_block_from_released`` maps them
   back onto exactly the drawn engine tensors (bitwise),
3. runs the reference block (and each of its ops alone) in fp32 on seeded inputs and
   writes the outputs to ``tests/golden/<case>.npz``.

``miniworld_engine`` is not installed anywhere; the legacy block reaches it only through
names it never calls on this path, so a stub module stands in for it at import time.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from foldforge_b200.synthetic import (  # noqa: E402
    EVOFORMER_PAIR_NAMES,
    BlockShape,
    block_state,
    evoformer_state,
    inputs,
    msa_inputs,
    dit_inputs,
    dit_stack_state,
)


def _stub_engine() -> None:
    engine = types.ModuleType("miniworld_engine")
    mods = types.ModuleType("miniworld_engine.modules")
    prim = types.ModuleType("miniworld_engine.modules.primitives")
    prim.MasterWeights = type("MasterWeights", (), {})
    mods.LayerNorm = torch.nn.LayerNorm
    for name in (
        "MSAPairWeightedAveraging", "OuterProductMean", "Transition", "TriangleAttention",
        "TriangleMultiplication", "PairformerBlock", "PairformerConfig",
    ):
        setattr(mods, name, type(name, (torch.nn.Module,), {}))
    mods.primitives = prim
    engine.modules = mods
    sys.modules.update({
        "miniworld_engine": engine,
        "miniworld_engine.modules": mods,
        "miniworld_engine.modules.primitives": prim,
    })


def released_from_engine(state: dict[str, torch.Tensor], g: torch.Generator) -> dict[str, torch.Tensor]:
    """Engine keys -> the legacy block's released keys (inverse of the converter)."""
    out: dict[str, torch.Tensor] = {}
    for dst, src, outgoing in (
        ("triangle_multiplication_outgoing", "tri_multi_outgoing", True),
        ("triangle_multiplication_incoming", "tri_multi_incoming", False),
    ):
        e = {k[len(src) + 1 :]: v for k, v in state.items() if k.startswith(src + ".")}
        # row 2k = branch a of hidden channel k, 2k+1 = branch b; incoming: left = b
        a, b = ("to_left", "to_right") if outgoing else ("to_right", "to_left")
        for released, engine in (("projection", ""), ("gate", "_gate")):
            pa, pb = e[f"{a}{engine}.weight"], e[f"{b}{engine}.weight"]
            out[f"{dst}.{released}.weight"] = torch.stack([pa, pb], 1).reshape(-1, pa.shape[1])
        out[f"{dst}.left_norm_input.weight"] = e["ln_pair.weight"]
        out[f"{dst}.left_norm_input.bias"] = e["ln_pair.bias"]
        out[f"{dst}.center_norm.weight"] = e["ln_out.weight"]
        out[f"{dst}.center_norm.bias"] = e["ln_out.bias"]
        out[f"{dst}.output_projection.weight"] = e["to_out.weight"]
        out[f"{dst}.gating_linear.weight"] = e["to_gate.weight"]
    for dst, src in (("pair_attention1", "tri_atten_starting"), ("pair_attention2", "tri_atten_ending")):
        for released, engine in (
            ("act_norm.weight", "ln_pair.weight"), ("act_norm.bias", "ln_pair.bias"),
            ("pair_bias_projection.weight", "to_bias.weight"), ("q_projection.weight", "to_query.weight"),
            ("k_projection.weight", "to_key.weight"), ("v_projection.weight", "to_value.weight"),
            ("gating_query.weight", "to_gate.weight"), ("output_projection.weight", "to_out.weight"),
        ):
            out[f"{dst}.{released}"] = state[f"{src}.{engine}"]
    for dst, src in (("pair_transition", "transition_pair"), ("single_transition", "single_transition")):
        if f"{src}.ln_in.weight" not in state:
            continue
        out[f"{dst}.input_layer_norm.weight"] = state[f"{src}.ln_in.weight"]
        out[f"{dst}.input_layer_norm.bias"] = state[f"{src}.ln_in.bias"]
        out[f"{dst}.transition1.weight"] = torch.cat([state[f"{src}.expand_a.weight"], state[f"{src}.expand_b.weight"]], 0)
        out[f"{dst}.transition2.weight"] = state[f"{src}.squeeze.weight"]
    if "single_attention.to_query.weight" in state:
        sa = "single_attention_"
        out[f"{sa}.adaptive_layernorm.layer_norm.weight"] = state["single_attention.ln_single.weight"]
        out[f"{sa}.adaptive_layernorm.layer_norm.bias"] = state["single_attention.ln_single.bias"]
        out[f"{sa}.q_projection.weight"] = state["single_attention.to_query.weight"]
        out[f"{sa}.q_projection.bias"] = state["single_attention.to_query.bias"]
        out[f"{sa}.k_projection.weight"] = state["single_attention.to_key.weight"]
        out[f"{sa}.v_projection.weight"] = state["single_attention.to_value.weight"]
        out[f"{sa}.gating_query.weight"] = state["single_attention.to_gate.weight"]
        out[f"{sa}.adaptive_zero_init.transition2.weight"] = state["single_attention.to_out.weight"]
        out["single_pair_logits_norm.weight"] = state["single_attention.ln_pair.weight"]
        # discarded by the converter (softmax-invariant): a NON-zero value here checks that
        out["single_pair_logits_norm.bias"] = 0.05 * torch.randn(state["single_attention.ln_pair.weight"].shape, generator=g)
        out["single_pair_logits_projection.weight"] = state["single_attention.to_bias.weight"]
    return out


def _digest(state: dict[str, torch.Tensor]) -> str:
    h = hashlib.sha256()
    for k in sorted(state):
        h.update(k.encode())
        h.update(state[k].contiguous().numpy().tobytes())
    return h.hexdigest()


def run_case(name: str, *, shape: BlockShape, n: int, masked: list[int], scheme: str, wseed: int,
             iseed: int, extra_bias: bool = False, keep_rows: list[int] | None = None) -> None:
    from foldforge.models.checkpoints.legacy.pairformer import PairformerBlock
    from foldforge.models.checkpoints.legacy.released import pairformer_block_from_released

    g = torch.Generator().manual_seed(wseed)
    state = block_state(g, shape, scheme)
    legacy = PairformerBlock(
        n_heads=shape.n_head_single, c_pair=shape.c_z, c_single=shape.c_s,
        n_heads_pair=shape.n_head_pair, num_intermediate_factor=shape.n_pair,
        single_intermediate_factor=shape.n_single,
    ).eval()
    legacy.load_state_dict(released_from_engine(state, torch.Generator().manual_seed(wseed + 1000)), strict=True)
    back = pairformer_block_from_released(legacy.state_dict())
    assert set(back) == set(state), sorted(set(back) ^ set(state))
    for k, v in state.items():
        assert torch.equal(back[k], v), k

    z, s, tokens = inputs(n, iseed, shape.c_z, shape.c_s)
    for t in masked:
        tokens[t] = 0
    pair_mask = tokens[:, None] * tokens[None, :]
    bias = torch.randn(n, n, generator=torch.Generator().manual_seed(iseed + 7)) if extra_bias else None
    with torch.no_grad():
        ops = {
            "tri_multi_outgoing": z + legacy.triangle_multiplication_outgoing(z, pair_mask),
            "tri_multi_incoming": z + legacy.triangle_multiplication_incoming(z, pair_mask),
            "tri_atten_starting": legacy.pair_attention1.residual(z, pair_mask),
            "tri_atten_ending": legacy.pair_attention2.residual(z, pair_mask),
            "transition_pair": z + legacy.pair_transition(z),
            "single_transition": s + legacy.single_transition(s),
        }
        pair_logits = legacy.single_pair_logits_projection(legacy.single_pair_logits_norm(z)).permute(2, 0, 1)
        if bias is not None:
            pair_logits = pair_logits + bias[None]
        ops["single_attention"] = s + legacy.single_attention_(s, tokens, pair_logits=pair_logits)
        out_pair, out_single = legacy(z.clone(), pair_mask, s.clone(), tokens, extra_pair_bias=bias)
    record: dict[str, np.ndarray] = {
        "n": np.array(n), "tokens": tokens.numpy(),
        "shape": np.array([shape.c_z, shape.c_s, shape.hidden_mul, shape.n_head_pair, shape.d_tri,
                           shape.n_head_single, shape.n_pair, shape.n_single]),
        "scheme": np.array(scheme), "wseed": np.array(wseed), "iseed": np.array(iseed),
        "weights_sha256": np.array(_digest(state)),
        "inputs_sha256": np.array(_digest({"z": z, "s": s})),
        "pair_sum": np.array(out_pair.double().sum().item()),
        "pair_sumsq": np.array(out_pair.double().square().sum().item()),
        "single_sum": np.array(out_single.double().sum().item()),
        "single_sumsq": np.array(out_single.double().square().sum().item()),
        "out_single": out_single.numpy(),
    }
    if bias is not None:
        record["extra_pair_bias"] = bias.numpy()
    if keep_rows is None:
        record["out_pair"] = out_pair.numpy()
        for k, v in ops.items():
            record[f"op.{k}"] = v.numpy()
    else:
        record["rows"] = np.array(keep_rows)
        record["out_pair_rows"] = out_pair[keep_rows].numpy()
    np.savez_compressed(HERE / f"{name}.npz", **record)
    print(f"{name}: N={n} masked={masked} -> {HERE / (name + '.npz')}")


def released_evoformer_from_engine(state: dict[str, torch.Tensor], g: torch.Generator) -> dict[str, torch.Tensor]:
    """Engine keys of an MSA-stack block -> the released ``EvoformerBlock`` keys (the inverse of
    ``evoformer_block_from_released``): the pair track through :func:`released_from_engine`, then
    the outer product mean, the pair-weighted averaging and the MSA transition."""
    back_names = {v: k for k, v in EVOFORMER_PAIR_NAMES.items()}
    pair_part = {}
    for key, value in state.items():
        head, rest = key.split(".", 1)
        if head in back_names:
            pair_part[f"{back_names[head]}.{rest}"] = value
    out = released_from_engine(pair_part, g)
    o = "outer_product_mean"
    out[f"{o}.layer_norm_input.weight"] = state[f"{o}.ln_msa.weight"]
    out[f"{o}.layer_norm_input.bias"] = state[f"{o}.ln_msa.bias"]
    out[f"{o}.left_projection.weight"] = state[f"{o}.to_left.weight"]
    out[f"{o}.right_projection.weight"] = state[f"{o}.to_right.weight"]
    w = state[f"{o}.to_out.weight"]  # [c_z, K K] = output_w.reshape(K K, c_z).T
    k = int(round(w.shape[1] ** 0.5))
    out[f"{o}.output_w"] = w.t().reshape(k, k, w.shape[0]).contiguous()
    out[f"{o}.output_b"] = state[f"{o}.to_out.bias"]
    a = "msa_attention1"
    out[f"{a}.act_norm.weight"] = state[f"{a}.ln_msa.weight"]
    out[f"{a}.act_norm.bias"] = state[f"{a}.ln_msa.bias"]
    out[f"{a}.pair_norm.weight"] = state[f"{a}.ln_pair.weight"]
    # discarded by the converter (softmax-invariant): a NON-zero value here checks that
    out[f"{a}.pair_norm.bias"] = 0.05 * torch.randn(state[f"{a}.ln_pair.weight"].shape, generator=g)
    out[f"{a}.pair_logits.weight"] = state[f"{a}.to_bias.weight"]
    out[f"{a}.v_projection.weight"] = state[f"{a}.to_value.weight"]
    out[f"{a}.gating_query.weight"] = state[f"{a}.to_gate.weight"]
    out[f"{a}.output_projection.weight"] = state[f"{a}.to_out.weight"]
    t = "msa_transition"
    out[f"{t}.input_layer_norm.weight"] = state[f"{t}.ln_in.weight"]
    out[f"{t}.input_layer_norm.bias"] = state[f"{t}.ln_in.bias"]
    out[f"{t}.transition1.weight"] = torch.cat([state[f"{t}.expand_a.weight"], state[f"{t}.expand_b.weight"]], 0)
    out[f"{t}.transition2.weight"] = state[f"{t}.squeeze.weight"]
    return out


def run_evoformer_case(name: str, *, n_seq: int, n: int, masked: int, scheme: str, wseed: int, iseed: int) -> None:
    """The reference's released-layout ``EvoformerBlock`` with AF3's spec on seeded engine-key
    weights (converter round trip checked bitwise) and seeded MSA / pair inputs."""
    from foldforge.models.checkpoints.legacy.pairformer import EvoformerBlock
    from foldforge.models.checkpoints.legacy.released import evoformer_block_from_released
    from foldforge.modules.dense.spec import ALPHAFOLD3

    state = evoformer_state(torch.Generator().manual_seed(wseed), scheme=scheme)
    legacy = EvoformerBlock(c_msa=64, c_pair=128, n_heads_pair=4, spec=ALPHAFOLD3).eval()
    legacy.load_state_dict(released_evoformer_from_engine(state, torch.Generator().manual_seed(wseed + 1000)),
                           strict=True)
    back = evoformer_block_from_released(legacy.state_dict())
    assert set(back) == set(state), sorted(set(back) ^ set(state))
    for k, v in state.items():
        assert torch.equal(back[k], v), k
    msa, z, msa_mask, tokens = msa_inputs(n_seq, n, iseed, masked_suffix=masked)
    pair_mask = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        opm = legacy.outer_product_mean(msa, msa_mask)
        pwa = legacy.msa_attention1.residual(msa, msa_mask, z)
        out_msa, out_pair = legacy(msa.clone(), z.clone(), msa_mask, pair_mask)
    record = {
        "n": np.array(n), "n_seq": np.array(n_seq), "masked": np.array(masked), "scheme": np.array(scheme),
        "wseed": np.array(wseed), "iseed": np.array(iseed), "weights_sha256": np.array(_digest(state)),
        "inputs_sha256": np.array(_digest({"msa": msa, "z": z, "msa_mask": msa_mask})),
        "op.outer_product_mean": opm.numpy(), "op.msa_attention1": pwa.numpy(),
        "out_msa": out_msa.numpy(), "out_pair": out_pair.numpy(),
    }
    np.savez_compressed(HERE / f"{name}.npz", **record)
    print(f"{name}: S={n_seq} N={n} masked={masked} -> {HERE / (name + '.npz')}")


def released_dit_from_engine(blocks: list[dict[str, torch.Tensor]], super_block_size: int) -> dict[str, torch.Tensor]:
    """Engine keys of AF3 token DiT blocks -> the released ``DiffusionTransformer`` keys (the
    inverse of ``token_dit_blocks_from_released``): one shared pair norm (every block's
    ``ln_pair`` must be the same tensor values), the blocks' ``to_bias`` stacked per super block
    into ``pair_logits_projection.<j>``, each block's attention / transition renamed."""
    out: dict[str, torch.Tensor] = {"pair_input_layer_norm.weight": blocks[0]["attention.ln_pair.weight"]}
    for j in range(len(blocks) // super_block_size):
        out[f"pair_logits_projection.{j}.weight"] = torch.cat(
            [blocks[j * super_block_size + t]["attention.to_bias.weight"] for t in range(super_block_size)], 0)

    def adaln(dst: str, src: str, st: dict[str, torch.Tensor]) -> None:
        out[f"{dst}.single_cond_layer_norm.weight"] = st[f"{src}.ln_cond.weight"]
        out[f"{dst}.single_cond_scale.weight"] = st[f"{src}.to_scale.weight"]
        out[f"{dst}.single_cond_scale.bias"] = st[f"{src}.to_scale.bias"]
        out[f"{dst}.single_cond_bias.weight"] = st[f"{src}.to_bias.weight"]

    for i, st in enumerate(blocks):
        a, t = f"self_attention.{i}", f"transition_block.{i}"
        adaln(f"{a}.adaptive_layernorm", "attention.ada_ln_in", st)
        out[f"{a}.q_projection.weight"] = st["attention.to_query.weight"]
        out[f"{a}.q_projection.bias"] = st["attention.to_query.bias"]
        out[f"{a}.k_projection.weight"] = st["attention.to_key.weight"]
        out[f"{a}.v_projection.weight"] = st["attention.to_value.weight"]
        out[f"{a}.gating_query.weight"] = st["attention.to_gate.weight"]
        out[f"{a}.adaptive_zero_init.transition2.weight"] = st["attention.to_out.weight"]
        out[f"{a}.adaptive_zero_init.adaptive_zero_cond.weight"] = st["attention.to_scale.weight"]
        out[f"{a}.adaptive_zero_init.adaptive_zero_cond.bias"] = st["attention.to_scale.bias"]
        adaln(f"{t}.adaptive_layernorm", "transition.ada_ln_in", st)
        out[f"{t}.transition1.weight"] = torch.cat([st["transition.expand_a.weight"], st["transition.expand_b.weight"]], 0)
        out[f"{t}.adaptive_zero_init.transition2.weight"] = st["transition.squeeze.weight"]
        out[f"{t}.adaptive_zero_init.adaptive_zero_cond.weight"] = st["transition.to_scale.weight"]
        out[f"{t}.adaptive_zero_init.adaptive_zero_cond.bias"] = st["transition.to_scale.bias"]
    return out


def run_dit_case(name: str, *, samples: int, n: int, masked: int, n_blocks: int, super_block_size: int,
                 scheme: str, wseed: int, iseed: int) -> None:
    """The reference's released-layout token ``DiffusionTransformer`` with AF3's spec on seeded
    engine-key weights (converter round trip checked bitwise) and seeded inputs."""
    from foldforge.models.checkpoints.legacy.released import token_dit_blocks_from_released
    from foldforge.models.checkpoints.legacy.transformer import DiffusionTransformer
    from foldforge.modules.dense.spec import ALPHAFOLD3

    blocks = dit_stack_state(n_blocks, wseed, scheme)
    legacy = DiffusionTransformer(c_act=768, c_single_cond=384, c_pair_cond=128, num_head=16, num_blocks=n_blocks,
                                  super_block_size=super_block_size, spec=ALPHAFOLD3).eval()
    legacy.load_state_dict(released_dit_from_engine(blocks, super_block_size), strict=True)
    back = token_dit_blocks_from_released(legacy.state_dict(), n_head=16, super_block_size=super_block_size)
    assert len(back) == n_blocks
    for got, want in zip(back, blocks, strict=True):
        assert set(got) == set(want), sorted(set(got) ^ set(want))
        for k, v in want.items():
            assert torch.equal(got[k], v), k
    x, cond, pair, mask = dit_inputs(samples, n, iseed, masked_suffix=masked)
    with torch.no_grad():
        pl = legacy.pair_logits_projection[0](legacy.pair_input_layer_norm(pair))
        pl0 = pl.reshape(n, n, super_block_size, 16)[:, :, 0].permute(2, 0, 1)
        att = legacy.self_attention[0](x, mask, pl0, cond)
        tr = legacy.transition_block[0](x + att, cond)
        out = legacy(x.clone(), mask, cond, pair)
    record = {
        "samples": np.array(samples), "n": np.array(n), "masked": np.array(masked), "n_blocks": np.array(n_blocks),
        "scheme": np.array(scheme), "wseed": np.array(wseed), "iseed": np.array(iseed),
        "weights_sha256": np.array(_digest({f"{i}.{k}": v for i, b in enumerate(blocks) for k, v in b.items()})),
        "inputs_sha256": np.array(_digest({"x": x, "cond": cond, "pair": pair, "mask": mask})),
        "op.attention0": att.numpy(), "op.transition0": tr.numpy(), "out": out.numpy(),
    }
    np.savez_compressed(HERE / f"{name}.npz", **record)
    print(f"{name}: S={samples} N={n} masked={masked} blocks={n_blocks} -> {HERE / (name + '.npz')}")


SMALL = BlockShape(c_z=32, c_s=64, hidden_mul=32, n_head_pair=4, d_tri=8, n_head_single=4, n_pair=4, n_single=4)
AF3 = BlockShape()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="the src/ directory of a FoldForge checkout (the package foldforge is imported from it)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    _stub_engine()
    torch.set_num_threads(8)
    # the reference test's own case: AF3 widths, 24 tokens, last 3 masked
    run_case("af3_n24_masked3", shape=AF3, n=24, masked=[21, 22, 23], scheme="randomise", wseed=1, iseed=0)
    # benchmark configuration 1 (N=128, all tokens real, N(0, 0.02) weights), rows kept
    run_case("af3_n128_config1", shape=AF3, n=128, masked=[], scheme="baseline", wseed=0, iseed=0,
             keep_rows=[0, 37, 127])
    # small widths: ragged length, interior + suffix padding, extra pair bias
    run_case("small_n13_ragged", shape=SMALL, n=13, masked=[3, 7, 11, 12], scheme="randomise", wseed=2, iseed=3,
             extra_bias=True)
    # every token masked: uniform attention rows, zero contraction
    run_case("small_n5_allmasked", shape=SMALL, n=5, masked=[0, 1, 2, 3, 4], scheme="randomise", wseed=4, iseed=5)
    # a single token
    run_case("small_n1", shape=SMALL, n=1, masked=[], scheme="randomise", wseed=6, iseed=7)
    # the MSA-stack block (AF3): the reference test's shape (6 MSA rows, 20 tokens, 3 padded)
    # and benchmark configuration 4's weight scheme at a small size
    run_evoformer_case("evo_s6_n20_masked3", n_seq=6, n=20, masked=3, scheme="randomise", wseed=8, iseed=9)
    run_evoformer_case("evo_s33_n40_baseline", n_seq=33, n=40, masked=2, scheme="baseline", wseed=10, iseed=11)
    # the token diffusion transformer (AF3 widths: 768 / 16 heads, 384 conditioning, 128 pair):
    # two samples over 24 tokens with 3 padded, and one sample over 40 tokens through a whole
    # super block of four
    run_dit_case("dit_s2_n24_masked3", samples=2, n=24, masked=3, n_blocks=2, super_block_size=2,
                 scheme="randomise", wseed=12, iseed=13)
    run_dit_case("dit_s1_n40_sb4", samples=1, n=40, masked=0, n_blocks=4, super_block_size=4,
                 scheme="randomise", wseed=14, iseed=15)


if __name__ == "__main__":
    main()
