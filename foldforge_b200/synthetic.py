"""Seeded synthetic weights and inputs for the Pairformer block (no checkpoints here).

Weights are produced directly in the ENGINE state-dict schema, the one
``pairformer_block_from_released`` (``legacy/released.py:318-369``) emits: 56 tensors per
AF3 block. Keys are drawn in the fixed order of :func:`block_schema` from ONE
``torch.Generator``; a trunk draws its blocks in order from the same generator.

Schemes:

* ``"baseline"``: every matrix and every non-LayerNorm bias ``~N(0, 0.02)``, LayerNorm
  gamma 1 and beta 0 (the benchmark configurations).
* ``"randomise"``: the reference test's ``randomise`` (``tests/models/test_engine_graph.py:
  40-51``): matrices ``0.08 N(0,1)``, norm weights ``1 + 0.1 N``, other vectors
  ``0.05 N`` -- a non-trivial LayerNorm affine for parity work.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

Tensor = torch.Tensor


@dataclass(frozen=True)
class BlockShape:
    """Widths of one AF3 Pairformer block (defaults: ``modules/dense/spec.py:18-25,161``)."""

    c_z: int = 128
    c_s: int = 384
    hidden_mul: int = 128
    n_head_pair: int = 4
    d_tri: int = 32
    n_head_single: int = 16
    n_pair: int = 4
    n_single: int = 4


def block_schema(shape: BlockShape = BlockShape(), single: bool = True) -> list[tuple[str, tuple[int, ...]]]:
    """``[(engine key, shape)]`` of one block, in the converter's output order."""
    c, cs, h = shape.c_z, shape.c_s, shape.hidden_mul
    ht = shape.n_head_pair * shape.d_tri
    out: list[tuple[str, tuple[int, ...]]] = []
    for name in ("tri_multi_outgoing", "tri_multi_incoming"):
        out += [
            (f"{name}.ln_pair.weight", (c,)),
            (f"{name}.ln_pair.bias", (c,)),
            (f"{name}.ln_out.weight", (h,)),
            (f"{name}.ln_out.bias", (h,)),
            (f"{name}.to_left.weight", (h, c)),
            (f"{name}.to_right.weight", (h, c)),
            (f"{name}.to_left_gate.weight", (h, c)),
            (f"{name}.to_right_gate.weight", (h, c)),
            (f"{name}.to_out.weight", (c, h)),
            (f"{name}.to_gate.weight", (c, c)),
        ]
    for name in ("tri_atten_starting", "tri_atten_ending"):
        out += [
            (f"{name}.ln_pair.weight", (c,)),
            (f"{name}.ln_pair.bias", (c,)),
            (f"{name}.to_bias.weight", (shape.n_head_pair, c)),
            (f"{name}.to_query.weight", (ht, c)),
            (f"{name}.to_key.weight", (ht, c)),
            (f"{name}.to_value.weight", (ht, c)),
            (f"{name}.to_gate.weight", (ht, c)),
            (f"{name}.to_out.weight", (c, ht)),
        ]
    out += [
        ("transition_pair.ln_in.weight", (c,)),
        ("transition_pair.ln_in.bias", (c,)),
        ("transition_pair.expand_a.weight", (shape.n_pair * c, c)),
        ("transition_pair.expand_b.weight", (shape.n_pair * c, c)),
        ("transition_pair.squeeze.weight", (c, shape.n_pair * c)),
    ]
    if single:
        out += [
            ("single_attention.ln_single.weight", (cs,)),
            ("single_attention.ln_single.bias", (cs,)),
            ("single_attention.to_query.weight", (cs, cs)),
            ("single_attention.to_query.bias", (cs,)),
            ("single_attention.to_key.weight", (cs, cs)),
            ("single_attention.to_value.weight", (cs, cs)),
            ("single_attention.ln_pair.weight", (c,)),
            ("single_attention.to_bias.weight", (shape.n_head_single, c)),
            ("single_attention.to_gate.weight", (cs, cs)),
            ("single_attention.to_out.weight", (cs, cs)),
            ("single_transition.ln_in.weight", (cs,)),
            ("single_transition.ln_in.bias", (cs,)),
            ("single_transition.expand_a.weight", (shape.n_single * cs, cs)),
            ("single_transition.expand_b.weight", (shape.n_single * cs, cs)),
            ("single_transition.squeeze.weight", (cs, shape.n_single * cs)),
        ]
    return out


def _is_norm(key: str) -> bool:
    return ".ln_" in key


def block_state(
    generator: torch.Generator,
    shape: BlockShape = BlockShape(),
    scheme: str = "baseline",
    single: bool = True,
) -> dict[str, Tensor]:
    """One block's engine-key state dict (fp32), drawn from ``generator``."""
    if scheme not in ("baseline", "randomise"):
        raise ValueError(f"unknown weight scheme {scheme!r}")
    state: dict[str, Tensor] = {}
    for key, dims in block_schema(shape, single):
        noise = torch.randn(dims, generator=generator, dtype=torch.float32)
        if scheme == "baseline":
            if _is_norm(key):
                value = torch.ones(dims) if key.endswith("weight") else torch.zeros(dims)
            else:
                value = 0.02 * noise
        elif len(dims) > 1:
            value = 0.08 * noise
        elif _is_norm(key) and key.endswith("weight"):
            value = 1.0 + 0.1 * noise
        else:
            value = 0.05 * noise
        state[key] = value
    return state


def trunk_state(
    n_blocks: int, seed: int = 0, shape: BlockShape = BlockShape(), scheme: str = "baseline"
) -> list[dict[str, Tensor]]:
    """``n_blocks`` block states initialised in order from one seeded generator."""
    g = torch.Generator().manual_seed(seed)
    return [block_state(g, shape, scheme) for _ in range(n_blocks)]


def inputs(
    n: int,
    seed: int = 0,
    c_z: int = 128,
    c_s: int = 384,
    masked_suffix: int = 0,
) -> tuple[Tensor, Tensor, Tensor]:
    """``(z [N,N,c_z], s [N,c_s], tokens [N])``: ``z`` then ``s`` drawn ``~N(0,1)`` from a
    generator seeded ``seed``; the last ``masked_suffix`` tokens are padding (0)."""
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n, n, c_z, generator=g)
    s = torch.randn(n, c_s, generator=g)
    tokens = torch.ones(n)
    if masked_suffix:
        tokens[n - masked_suffix :] = 0
    return z, s, tokens


#: the Pairformer block's pair-track children under their names in the MSA-stack block
#: (``legacy/released.py:722-749``)
EVOFORMER_PAIR_NAMES = {
    "tri_multi_outgoing": "triangle_multiplication_outgoing",
    "tri_multi_incoming": "triangle_multiplication_incoming",
    "tri_atten_starting": "pair_attention1",
    "tri_atten_ending": "pair_attention2",
    "transition_pair": "pair_transition",
}


def evoformer_schema(c_m: int = 64, shape: BlockShape = BlockShape(), opm_hidden: int = 32, pwa_heads: int = 8,
                     n_msa: int = 4) -> list[tuple[str, tuple[int, ...]]]:
    """``[(engine key, shape)]`` of one AF3 MSA-stack block (``evoformer_block_from_released``):
    outer product mean, pair-weighted averaging, MSA transition, then the pair track."""
    c, k = shape.c_z, opm_hidden
    out: list[tuple[str, tuple[int, ...]]] = [
        ("outer_product_mean.ln_msa.weight", (c_m,)),
        ("outer_product_mean.ln_msa.bias", (c_m,)),
        ("outer_product_mean.to_left.weight", (k, c_m)),
        ("outer_product_mean.to_right.weight", (k, c_m)),
        ("outer_product_mean.to_out.weight", (c, k * k)),
        ("outer_product_mean.to_out.bias", (c,)),
        ("msa_attention1.ln_msa.weight", (c_m,)),
        ("msa_attention1.ln_msa.bias", (c_m,)),
        ("msa_attention1.ln_pair.weight", (c,)),
        ("msa_attention1.to_bias.weight", (pwa_heads, c)),
        ("msa_attention1.to_value.weight", (c_m, c_m)),
        ("msa_attention1.to_gate.weight", (c_m, c_m)),
        ("msa_attention1.to_out.weight", (c_m, c_m)),
        ("msa_transition.ln_in.weight", (c_m,)),
        ("msa_transition.ln_in.bias", (c_m,)),
        ("msa_transition.expand_a.weight", (n_msa * c_m, c_m)),
        ("msa_transition.expand_b.weight", (n_msa * c_m, c_m)),
        ("msa_transition.squeeze.weight", (c_m, n_msa * c_m)),
    ]
    for key, dims in block_schema(shape, single=False):
        head, rest = key.split(".", 1)
        out.append((f"{EVOFORMER_PAIR_NAMES[head]}.{rest}", dims))
    return out


def evoformer_state(generator: torch.Generator, c_m: int = 64, shape: BlockShape = BlockShape(),
                    scheme: str = "baseline") -> dict[str, Tensor]:
    """One MSA-stack block's engine-key state dict (fp32), drawn in schema order from ``generator``
    with the same schemes as :func:`block_state`."""
    if scheme not in ("baseline", "randomise"):
        raise ValueError(f"unknown weight scheme {scheme!r}")
    state: dict[str, Tensor] = {}
    for key, dims in evoformer_schema(c_m, shape):
        noise = torch.randn(dims, generator=generator, dtype=torch.float32)
        if scheme == "baseline":
            if _is_norm(key):
                value = torch.ones(dims) if key.endswith("weight") else torch.zeros(dims)
            else:
                value = 0.02 * noise
        elif len(dims) > 1:
            value = 0.08 * noise
        elif _is_norm(key) and key.endswith("weight"):
            value = 1.0 + 0.1 * noise
        else:
            value = 0.05 * noise
        state[key] = value
    return state


def msa_inputs(n_seq: int, n: int, seed: int = 0, c_m: int = 64, c_z: int = 128, masked_suffix: int = 0,
               row_dropout: float = 0.2) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """``(msa [S, N, c_m], z [N, N, c_z], msa_mask [S, N], tokens [N])`` from a generator seeded
    ``seed``: MSA then pair ~N(0, 1), each MSA position kept with probability ``1 - row_dropout``
    (the first row, the query sequence, always), padded tokens masked in every row."""
    g = torch.Generator().manual_seed(seed)
    msa = torch.randn(n_seq, n, c_m, generator=g)
    z = torch.randn(n, n, c_z, generator=g)
    tokens = torch.ones(n)
    if masked_suffix:
        tokens[n - masked_suffix:] = 0
    msa_mask = (torch.rand(n_seq, n, generator=g) > row_dropout).float() * tokens
    msa_mask[0] = tokens
    return msa, z, msa_mask, tokens


# ------------------------------------------------------------------------- diffusion transformer
def dit_schema(c: int = 768, c_cond: int = 384, c_pair: int = 128, n_head: int = 16,
               factor: int = 2) -> list[tuple[str, tuple[int, ...]]]:
    """Engine keys and shapes of one AF3 token DiT block (``TokenDiT``: the converter's
    ``legacy/released.py:372-509`` names): AdaLN + pair-biased attention, AdaLN + SwiGLU
    transition, each output gated by the conditioning."""

    def adaln(prefix: str) -> list[tuple[str, tuple[int, ...]]]:
        return [(f"{prefix}.ln_cond.weight", (c_cond,)), (f"{prefix}.to_scale.weight", (c, c_cond)),
                (f"{prefix}.to_scale.bias", (c,)), (f"{prefix}.to_bias.weight", (c, c_cond))]

    return [
        *adaln("attention.ada_ln_in"),
        ("attention.to_query.weight", (c, c)), ("attention.to_query.bias", (c,)),
        ("attention.to_key.weight", (c, c)), ("attention.to_value.weight", (c, c)),
        ("attention.to_gate.weight", (c, c)),
        ("attention.to_scale.weight", (c, c_cond)), ("attention.to_scale.bias", (c,)),
        ("attention.to_out.weight", (c, c)),
        ("attention.ln_pair.weight", (c_pair,)), ("attention.to_bias.weight", (n_head, c_pair)),
        *adaln("transition.ada_ln_in"),
        ("transition.expand_a.weight", (factor * c, c)), ("transition.expand_b.weight", (factor * c, c)),
        ("transition.squeeze.weight", (c, factor * c)),
        ("transition.to_scale.weight", (c, c_cond)), ("transition.to_scale.bias", (c,)),
    ]


def dit_state(generator: torch.Generator, scheme: str = "randomise", **dims: int) -> dict[str, Tensor]:
    """One token DiT block's engine-key state (fp32) drawn in schema order from ``generator``:
    ``baseline`` = N(0, 0.02) matrices, unit norm weights, zero biases; ``randomise`` =
    N(0, 0.05) matrices, norm weights 1 + N(0, 0.1), biases N(0, 0.5) (so the sigmoid gates
    are away from one half)."""
    if scheme not in ("baseline", "randomise"):
        raise ValueError(f"unknown weight scheme {scheme!r}")
    state: dict[str, Tensor] = {}
    for key, shape in dit_schema(**dims):
        noise = torch.randn(shape, generator=generator, dtype=torch.float32)
        norm = ".ln_" in key
        if scheme == "baseline":
            value = (torch.ones(shape) if norm else torch.zeros(shape)) if len(shape) == 1 else 0.02 * noise
        elif len(shape) > 1:
            value = 0.05 * noise
        else:
            value = 1.0 + 0.1 * noise if norm else 0.5 * noise
        state[key] = value
    return state


def dit_inputs(samples: int, n: int, seed: int = 0, c: int = 768, c_cond: int = 384, c_pair: int = 128,
               masked_suffix: int = 0) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """``(x [S, N, c], cond [N, c_cond], pair [N, N, c_pair], mask [N])`` from a generator seeded
    ``seed``: token activations, single and pair conditioning ~ N(0, 1), the last
    ``masked_suffix`` tokens padding."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(samples, n, c, generator=g)
    cond = torch.randn(n, c_cond, generator=g)
    pair = torch.randn(n, n, c_pair, generator=g)
    mask = torch.ones(n)
    if masked_suffix:
        mask[n - masked_suffix:] = 0
    return x, cond, pair, mask


def dit_stack_state(n_blocks: int, seed: int = 0, scheme: str = "randomise") -> list[dict[str, Tensor]]:
    """``n_blocks`` token DiT block states from one generator seeded ``seed``, every block with
    block 0's pair norm (AF3's token transformer has one shared pair norm)."""
    g = torch.Generator().manual_seed(seed)
    blocks = [dit_state(g, scheme) for _ in range(n_blocks)]
    for b in blocks[1:]:
        b["attention.ln_pair.weight"] = blocks[0]["attention.ln_pair.weight"].clone()
    return blocks
