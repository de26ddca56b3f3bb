"""The torch.library operators that let torch.compile trace the
orthogonalizers without graph breaks: schemas, the table encoding and the
fake (shape-only) implementations, all without a GPU."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import polar_switch
from polar_switch import coefficients, torch_ops


def test_operators_are_registered_with_their_schemas():
    ops = torch.ops.polar_switch
    import re
    mutated = re.compile(r"Tensor\(a\d*!\) out")
    assert mutated.search(str(ops.gram_out.default._schema))
    assert mutated.search(str(ops.square_out.default._schema))
    for name in ("circuit", "gns", "normalize", "apply"):
        assert "->" in str(getattr(ops, name).default._schema)


@pytest.mark.parametrize("method", [m for m in polar_switch.METHODS if m != "GNS"])
def test_table_encoding_round_trips(method):
    table = getattr(coefficients, method)
    lists = torch_ops.table_to_lists(table)
    back = torch_ops._lists_to_table(*lists)
    assert len(back) == len(table)
    for (r0, s0), (r1, s1) in zip(table, back):
        assert r0 == r1 and len(s0) == len(s1)
        for a, b in zip(s0, s1):
            assert tuple(a[:3]) == tuple(b[:3]) and all(float(x) == y for x, y in zip(a[3:], b[3:]))


def test_fake_implementations_describe_outputs():
    table = coefficients.PS3_55
    lists = torch_ops.table_to_lists(table)
    with FakeTensorMode():
        X = torch.empty(3, 256, 768, device="cuda", dtype=torch.bfloat16)
        Y = torch.ops.polar_switch.circuit(X, *lists, 3, 1e-7)
        assert Y.shape == X.shape and Y.dtype == X.dtype and Y.device == X.device
        G = torch.ops.polar_switch.gns(X, [1.0, 0.0, 0.0], [2], 1e-7)
        assert G.shape == X.shape and G.dtype == X.dtype
        Xh = torch.ops.polar_switch.normalize(X, 1e-7)
        assert Xh.shape == X.shape and Xh.dtype == torch.float16
        A = torch.empty(3, 256, 256, device="cuda", dtype=torch.float16)
        out = torch.empty_like(A)
        assert torch.ops.polar_switch.gram_out(Xh, False, out) is None
        assert torch.ops.polar_switch.square_out(A, out, None, 1.0, 0.0, 0.0, True) is None
        Xn = torch.ops.polar_switch.apply(Xh, A, False, 0.5)
        assert Xn.shape == X.shape and Xn.dtype == torch.float16
