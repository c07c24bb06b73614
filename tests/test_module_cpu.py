"""CPU: the module surface (README.md:6-68) and the rotary-table object."""
import math

import torch

from memory_efficient_attn_layer_b200 import CausalSoftmaxAttention, Yarn
from oracle.eager import rotary, yarn_tables


def test_module_init_matches_reference():
    torch.manual_seed(0)
    m = CausalSoftmaxAttention(256, 4, 32)
    bound = 0.5 / math.sqrt(256)
    for p in (m.q_proj, m.k_proj, m.v_proj, m.g_proj):
        assert p.weight.shape == (128, 256) and p.bias is None
        assert p.weight.abs().max() <= bound
    assert m.o_proj.weight.shape == (256, 128) and torch.count_nonzero(m.o_proj.weight) == 0


def test_yarn_tables_match_oracle_standin():
    y = Yarn(32, 64, dtype=torch.float32)
    f1, f2 = yarn_tables(32, 64)
    assert torch.allclose(y.factor1, f1, atol=1e-6) and torch.allclose(y.factor2, f2, atol=1e-6)


def test_yarn_rotary_matches_table_form():
    y = Yarn(16, 32, dtype=torch.float32)
    x = torch.randn(2, 32, 3, 16)
    want = rotary(x, y.factor1.view(1, 32, 1, 16), y.factor2.view(1, 32, 1, 16))
    assert torch.allclose(y.rotary(x), want, atol=1e-6)


def test_yarn_scaling_interpolates_low_frequencies():
    base = Yarn(64, 128, dtype=torch.float64)
    ext = Yarn(64, 128, scale=4.0, original_max_seq=4096, dtype=torch.float64)
    # pair magnitude = mscale = 0.1 ln 4 + 1
    mag = (ext.factor1[:, ::2] ** 2 + ext.factor2[:, ::2] ** 2).sqrt()
    assert torch.allclose(mag, torch.full_like(mag, 0.1 * math.log(4.0) + 1.0), atol=1e-9)
    # highest-frequency pair untouched, lowest-frequency pair slowed down by the scale
    ang = lambda t: torch.atan2(t.factor2[1, 1::2], t.factor1[1, ::2])
    assert math.isclose(float(ang(ext)[0]), float(ang(base)[0]), rel_tol=1e-9)
    assert math.isclose(float(ang(ext)[-1]), float(ang(base)[-1]) / 4.0, rel_tol=1e-6)


def test_yarn_frequencies_match_published_implementation():
    """YaRN "NTK-by-parts" frequencies and attention factor pinned to the YaRN
    implementation shipped in transformers (modeling_rope_utils._compute_yarn_parameters):
    same correction range (floor/ceil of the pair-index coordinates of beta_fast and
    beta_slow rotations over the original context), same linear ramp in the pair
    index, same magnitude 0.1 ln(scale) + 1."""
    import pytest

    tr = pytest.importorskip("transformers")
    from transformers.modeling_rope_utils import _compute_yarn_parameters

    for head_dim, scale, orig, base, bf, bs in [(64, 4.0, 2048, 10000.0, 32.0, 1.0), (128, 8.0, 4096, 500000.0, 32.0, 1.0),
                                                (32, 2.0, 1024, 10000.0, 16.0, 2.0)]:
        cfg = tr.LlamaConfig(hidden_size=head_dim * 4, num_attention_heads=4, head_dim=head_dim,
                             max_position_embeddings=int(orig * scale),
                             rope_parameters={"rope_type": "yarn", "rope_theta": base, "factor": scale,
                                              "original_max_position_embeddings": orig, "beta_fast": bf,
                                              "beta_slow": bs})
        want_inv, want_att = _compute_yarn_parameters(cfg)
        y = Yarn(head_dim, 64, base=base, scale=scale, original_max_seq=orig, beta_fast=bf, beta_slow=bs,
                 dtype=torch.float32)
        assert torch.allclose(y.inv_freq.float(), want_inv.float(), rtol=2e-6, atol=0), (head_dim, scale)
        assert math.isclose(y.mscale, want_att, rel_tol=1e-12)
