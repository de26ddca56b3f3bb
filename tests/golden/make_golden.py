"""Generate the golden fixtures in tests/golden/ from the reference implementation.

Run in the build container, where the reference project is available:

    python tests/golden/make_golden.py --reference /path/to/polar-switch

It reads the reference's certified circuits (coefficient_search/stage*.json)
and imports the reference package to run its own code on CPU:
  * the Triton backend (polar_switch/triton_kernels.py) under
    TRITON_INTERPRET=1 -- the kernel the reference uses whenever QuACK does
    not apply, evaluated by Triton's CPU interpreter;
  * the reference evaluator _run (polar_switch/__init__.py:25-45) with that
    backend, for whole circuits;
  * the reference CPU fallback (make_polynomial_orthogonalizer(...)(X_cpu),
    which runs POLAR_EXPRESS through torch.bmm, polar_switch/__init__.py:180-182);
  * the reference GNS recurrence with its PyTorch backend
    (polar_switch/gram_newton_schulz.py:75-122).

Inputs are seeded and stored next to the outputs, so the fixtures do not
depend on any random number generator at test time. The GPU box never runs
this script; the tests only read the .npz files it writes.
"""

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def certified(reference):
    """certified_circuits.json: the two circuits the reference certified with
    interval arithmetic (coefficient_search/stage1.json, stage2.json; PS2-64's
    outer iterations), as coefficient-table steps (w, i, r, a, b, c) with the
    buffers A = 0 and B = 1, and their certified intervals."""
    import json
    buf = {"A": 0, "B": 1}
    out = {}
    for stage in ("stage1", "stage2"):
        with open(os.path.join(reference, "coefficient_search", stage + ".json")) as f:
            d = json.load(f)
        assert d["status"] == "verified" and d["format"] == "two-buffer-iteration-v2"
        out[stage] = {
            "input_interval": d["input_interval"],
            "output_interval": d["output_interval"],
            "exact_intervals": d["exact_intervals"],
            "safety_factor": d["safety_factor"],
            "centered": d["centered"],
            "steps": [[buf[s["write"]], buf[s["square"]], buf[s["addend"]], s["a"], s["b"], s["c"]]
                      for s in d["iteration"]["steps"]],
        }
    with open(os.path.join(HERE, "certified_circuits.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote certified_circuits.json")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference project")
    ap.add_argument("--only", choices=["all", "certified", "circuits", "gns"], default="all",
                    help="'certified' writes certified_circuits.json alone; 'circuits' the whole-circuit "
                         "fixtures alone; 'gns' the GNS fixtures alone")
    ap.add_argument("--missing", action="store_true",
                    help="write only fixtures that do not exist yet (existing files stay byte for byte)")
    args = ap.parse_args()
    if args.only in ("all", "certified"):
        certified(os.path.abspath(args.reference))
    if args.only == "certified":
        return
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    import polar_switch as ref
    from polar_switch import coefficients, triton_kernels
    from polar_switch import gram_newton_schulz as gns

    def randn(shape, seed, scale=1.0):
        g = torch.Generator().manual_seed(seed)
        return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).float()

    def normalized(shape, seed):
        X = randn(shape, seed)
        return (X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)).half().contiguous()

    def save(name, **arrays):
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **{k: v.numpy() if hasattr(v, "numpy") else np.asarray(v)
                                     for k, v in arrays.items()})
        print("wrote", path)

    def exists(name):
        return args.missing and os.path.exists(os.path.join(HERE, name))

    # ---- whole circuits through the reference evaluator and Triton backend
    cases = [
        ("PS2_55", (1, 128, 256), 10),
        ("PS3_55", (1, 128, 256), 11),
        ("POLAR_EXPRESS", (1, 128, 256), 12),
        ("JORDAN", (1, 128, 256), 13),
        ("PS2_55", (2, 192, 64), 14),
        ("PS3_55", (1, 96, 96), 15),
        ("PS2_512", (1, 64, 160), 16),
        ("PS2_64", (1, 128, 256), 30),
        ("PS2_54", (1, 128, 256), 31),
        ("PS2_4111", (1, 128, 256), 32),
        ("PS2_11111", (1, 128, 256), 33),
        ("PS3_64", (1, 128, 256), 34),
        ("PS3_54", (1, 128, 256), 35),
    ]
    for method, shape, seed in cases:
        name = f"circuit_{method}_{'x'.join(map(str, shape))}"
        if exists(name + ".npz"):
            continue
        table = getattr(coefficients, method)
        nbuf = 1 + max(max(w, i, r) for _, steps in table for w, i, r, *_ in steps)
        Xc = randn(shape, seed)
        Y = ref._run(Xc, table, triton_kernels, 1e-7, nbuf)
        save(name, x=Xc, out=Y)
    if args.only == "circuits":
        return
    if args.only == "gns":
        gns_fixtures(args, randn, save, exists, gns)
        return

    # ---- the coefficient data (tables and GNS preset) of the reference
    import json
    names = [n for n in ref.METHODS if n != "GNS"]
    data = {"tables": {n: getattr(coefficients, n) for n in names},
            "gns": [list(c) for c in gns.GNS_COEFFICIENTS],
            "gns_polar_express": [list(c) for c in gns.POLAR_EXPRESS_COEFFICIENTS]}
    with open(os.path.join(HERE, "coefficients.json"), "w") as f:
        json.dump(data, f, indent=1)
    print("wrote coefficients.json")

    # ---- single operations of the Triton backend
    X = normalized((2, 128, 192), 1)
    G = torch.empty(2, 128, 128, dtype=torch.float16)
    triton_kernels.gram(X, False, G)
    save("op_gram_wide", x=X, out=G)

    Xt = normalized((2, 160, 96), 2)
    Gt = torch.empty(2, 96, 96, dtype=torch.float16)
    triton_kernels.gram(Xt, True, Gt)
    save("op_gram_tall", x=Xt, out=Gt)

    A = G.clone()
    C = torch.empty_like(A)
    triton_kernels.gram(normalized((2, 128, 192), 3), False, C)
    out = torch.empty_like(A)
    triton_kernels.square(A, C, out, 1.75, -0.6, 0.37)
    save("op_square", a=A, c=C, out=out, alpha=1.75, beta=-0.6, diag=0.37)

    C2 = C.clone()
    triton_kernels.square(A, C2, C2, 164.07644513428048, 49.58061223879703, 0.000500089059050944)
    save("op_square_inplace", a=A, c=C, out=C2, alpha=164.07644513428048,
         beta=49.58061223879703, diag=0.000500089059050944)

    for tall, seed in ((False, 4), (True, 5)):
        Xa = normalized((2, 96, 160) if not tall else (2, 160, 96), seed)
        B = G[:, :96, :96].contiguous()
        for residual in (0.0, 3.4445):
            Y = triton_kernels.apply(Xa, B, tall, residual)
            save(f"op_apply_{'tall' if tall else 'wide'}_{'res' if residual else 'nores'}",
                 x=Xa, b=B, out=Y, residual=residual)

    # ---- the reference CPU path: requested PS2_55, runs POLAR_EXPRESS in torch
    import warnings
    Xcpu = randn((128, 256), 20)
    polar = ref.make_polynomial_orthogonalizer("PS2_55", compile=False)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        Ycpu = polar(Xcpu)
    assert polar.last_execution["effective"] == "POLAR_EXPRESS"
    save("cpu_path_ps2_55_128x256", x=Xcpu, out=Ycpu)

    gns_fixtures(args, randn, save, exists, gns)


def gns_fixtures(args, randn, save, exists, gns):
    """GNS recurrence with the reference's PyTorch backend (rectangular):
    wide (X Xᵀ) and tall (XᵀX) inputs."""
    inst = gns.GramNewtonSchulz(ns_epsilon=1e-7, ns_use_kernels=False,
                                ns_coefficients=gns.GNS_COEFFICIENTS,
                                gram_newton_schulz_reset_iterations=[2], compile_kwargs=None)
    for shape, seed in (((2, 96, 224), 21), ((2, 224, 96), 22), ((1, 64, 320), 23)):
        name = f"gns_torch_{'x'.join(map(str, shape))}"
        if exists(name + ".npz"):
            continue
        Xg = randn(shape, seed)
        save(name, x=Xg, out=inst._select_gram(Xg))


if __name__ == "__main__":
    main()
