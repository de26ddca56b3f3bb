"""Host-side behaviour of the drop-in API (no GPU needed): method resolution,
table validation and error paths mirror the reference
(polar_switch/__init__.py:78-186); there is no CPU fallback."""

import math

import pytest
import torch

import polar_switch
from polar_switch import coefficients, circuit_flops, make_polynomial_orthogonalizer


def test_methods_tuple():
    assert polar_switch.METHODS == ("JORDAN", "POLAR_EXPRESS", "GNS", "PS2_55", "PS2_64", "PS2_54",
                                    "PS2_512", "PS2_4111", "PS2_11111", "PS3_55", "PS3_64", "PS3_54")
    for m in polar_switch.METHODS:
        if m != "GNS":
            assert isinstance(getattr(coefficients, m), tuple)


@pytest.mark.parametrize("method,buffers", [("PS2_55", 2), ("ps3_55", 3), ("POLAR_EXPRESS", 2),
                                            ("JORDAN", 2), ("PS2_512", 2), ("PS3_64", 3)])
def test_resolution_and_buffers(method, buffers):
    p = make_polynomial_orthogonalizer(method)
    assert p.buffers == buffers
    assert p.method == method.upper()
    assert p.fallback_events == [] and p.last_execution is None


def test_custom_table_name_lookup():
    p = make_polynomial_orthogonalizer(coefficients.PS2_55)
    assert p.method == "PS2_55"
    table = ((0.5, ((1, 0, 0, 1.0, -0.5, 0.25),)),)
    assert make_polynomial_orthogonalizer(table).method == "CUSTOM"


def test_unknown_method():
    with pytest.raises(ValueError, match="Unknown method"):
        make_polynomial_orthogonalizer("PS9_99")


@pytest.mark.parametrize("table", [
    (),                                                    # empty circuit
    ((0.0, ()),),                                          # outer iteration without steps
    ((math.inf, ((1, 0, 0, 1.0, 1.0, 0.0),)),),            # non-finite residual
    ((0.0, ((0, 0, 0, 1.0, 1.0, 0.0),)),),                 # dst == src
    ((0.0, ((1, 2, 0, 1.0, 1.0, 0.0),)),),                 # src not initialised
    ((0.0, ((1, 0, 2, 1.0, 1.0, 0.0),)),),                 # add not initialised
    ((0.0, ((1, 0, 0, math.nan, 1.0, 0.0),)),),            # non-finite coefficient
    ((0.0, ((1.0, 0, 0, 1.0, 1.0, 0.0),)),),               # non-integer index
    ((0.0, ((-1, 0, 0, 1.0, 1.0, 0.0),)),),                # negative index
])
def test_invalid_tables(table):
    with pytest.raises(ValueError):
        make_polynomial_orthogonalizer(table)


@pytest.mark.parametrize("eps", [0.0, -1.0, math.inf, math.nan])
def test_invalid_epsilon(eps):
    with pytest.raises(ValueError):
        make_polynomial_orthogonalizer("PS2_55", epsilon=eps)
    with pytest.raises(ValueError):
        make_polynomial_orthogonalizer("GNS", epsilon=eps)


def test_buffer_indices_written_earlier_in_same_outer_iteration_only():
    # B[1] written in outer 1 is not initialised at the start of outer 2
    table = ((0.0, ((1, 0, 0, 1.0, 1.0, 0.0),)), (0.0, ((2, 1, 0, 1.0, 1.0, 0.0),)))
    with pytest.raises(ValueError):
        make_polynomial_orthogonalizer(table)


@pytest.mark.parametrize("bad", [torch.zeros(5), torch.zeros(0, 4), torch.zeros(3, 4, dtype=torch.int32)])
def test_bad_inputs(bad):
    with pytest.raises(ValueError, match="Expected nonempty real matrices"):
        make_polynomial_orthogonalizer("PS2_55")(bad)
    with pytest.raises(ValueError, match="Expected nonempty real matrices"):
        make_polynomial_orthogonalizer("GNS")(bad)


def test_cpu_tensor_raises_instead_of_falling_back():
    p = make_polynomial_orthogonalizer("PS2_55")
    with pytest.raises(NotImplementedError, match="CUDA"):
        p(torch.randn(8, 16))
    assert p.fallback_events == [] and p.last_execution is None


def test_cuda_ops_reject_cpu_tensors():
    from polar_switch import cuda_ops
    X = torch.randn(8, 16).half()
    with pytest.raises(NotImplementedError):
        cuda_ops.gram(X, False, torch.empty(8, 8).half())
    with pytest.raises(NotImplementedError):
        cuda_ops.normalize(X, 1e-7)


def test_flop_counts_match_reference_formulas():
    n = 1024
    for alpha in (1, 2, 4):
        m = alpha * n
        assert circuit_flops(coefficients.PS2_55, n, m) == (6 * alpha + 10) * n ** 3
        assert circuit_flops(coefficients.PS3_55, m, n) == (6 * alpha + 10) * n ** 3
        assert circuit_flops(coefficients.POLAR_EXPRESS, n, m) == (15 * alpha + 5) * n ** 3
        assert circuit_flops(coefficients.PS2_512, n, m) == (9 * alpha + 8) * n ** 3
    from polar_switch.gram_newton_schulz import gns_flops
    assert gns_flops(1024, 4096) == (6 * 4 + 14) * 1024 ** 3


def test_qwen_step_flops():
    from polar_switch.distributed import qwen3_0_6b_banks
    total = sum(L * circuit_flops(coefficients.PS2_55, r, c) for L, r, c in qwen3_0_6b_banks())
    assert total == pytest.approx(4.81e12, rel=2e-3)
    assert sum(L for L, _, _ in qwen3_0_6b_banks()) == 196


def test_muon_module_groups_parameters_on_cpu():
    """The Muon optimizer's parameter grouping follows the reference and its
    kernel path refuses CPU tensors (there is no CPU fallback)."""
    from polar_switch.muon import muon_directions, parameter_groups

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = torch.nn.Embedding(10, 8)
            self.q_proj = torch.nn.Linear(8, 16, bias=True)
            self.o_proj = torch.nn.Linear(16, 8, bias=False)

    groups, scalars = parameter_groups(Block())
    assert [g["role"] for g in groups] == ["o_proj", "q_proj"]
    n_matrix = sum(len(g["params"]) for g in groups)
    assert n_matrix == 2 and len(scalars) == 2  # embedding + q_proj bias
    with pytest.raises(NotImplementedError):
        muon_directions([torch.zeros(4, 4)], [torch.zeros(4, 4)], 0.9, torch.bfloat16)
