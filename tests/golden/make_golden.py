"""Generates the golden fixtures in this directory by running the reference itself.

Run in a container where the reference source is available:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py [--reference-src PATH]

Each ``*.npz`` holds a case's inputs (or the numpy seed that regenerates them),
the reference's outputs and its autograd gradients, computed with the
reference's own CPU PyTorch algebra (the path ``TensorProduct``/``UvuTensorProduct``
take on CPU) in float64 and, where noted, float32.  ``cg_tables.npz`` holds the
reference's dense normalised CG tensors for every path up to m_max = 8.

Tests read only the ``.npz`` files; nothing at test time imports the reference.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _torch():
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    return torch


def _tp_case(name, channels, m_max, parity, normalization, rows, seed, cotangent, dtype,
             torch_rows=None, keep_rows=None):
    """TensorProduct case.  Weights come from the reference's seeded init
    (torch.manual_seed(seed) then the constructor); inputs are torch.randn in the
    order of the BASELINE recipe when ``torch_rows`` is given, else numpy."""
    torch = _torch()
    from ictc_o2_hp import TensorProduct
    torch.manual_seed(seed)
    tp = TensorProduct(channels, m_max, parity=parity, normalization=normalization)
    width = tp.representation_dimension
    record = {"channels": channels, "m_max": m_max, "parity": parity,
              "normalization": normalization, "seed": seed, "weight": tp.weight.detach().numpy()}
    if torch_rows is not None:
        x = torch.randn(torch_rows, width)
        y = torch.randn(torch_rows, width)
        record["torch_rows"] = torch_rows
    else:
        rng = np.random.default_rng(seed)
        x = torch.from_numpy(rng.standard_normal((rows, width)).astype(np.float32))
        y = torch.from_numpy(rng.standard_normal((rows, width)).astype(np.float32))
        record["x"], record["y"] = x.numpy(), y.numpy()
    n = x.shape[0]
    if cotangent == "ones":
        g = torch.ones(n, width)
    else:
        g = torch.from_numpy(np.random.default_rng(seed + 1).standard_normal(
            (n, width)).astype(np.float32))
        record["g"] = g.numpy()
    record["cotangent"] = cotangent
    for tag, dt in dtype:
        module = TensorProduct(channels, m_max, parity=parity, normalization=normalization)
        module = module.to(dt)
        # The reference computes in internal_compute_dtype (float32 by default,
        # native_o2.py:156, fast_o2.py:87-95) whatever the input dtype; the float64
        # arbiter must compute in float64 too.
        module.internal_compute_dtype = dt
        with torch.no_grad():
            module.weight.copy_(torch.from_numpy(record["weight"]).to(dt))
        xx, yy = x.to(dt).requires_grad_(True), y.to(dt).requires_grad_(True)
        out = module(xx, yy)
        dx, dy, dw = torch.autograd.grad(out, (xx, yy, module.weight), g.to(dt))
        arrays = {"out": out.detach(), "dx": dx, "dy": dy}
        for key, value in arrays.items():
            v = value.numpy()
            if keep_rows is not None:
                record[f"{key}_{tag}_rows"] = v[keep_rows]
                record[f"{key}_{tag}_sum"] = v.astype(np.float64).sum(axis=0)
            else:
                record[f"{key}_{tag}"] = v
        record[f"dw_{tag}"] = dw.numpy()
    if keep_rows is not None:
        record["keep_rows"] = np.asarray(keep_rows)
    record["paths"] = np.array([str(p) for p in module.paths])
    np.savez_compressed(HERE / f"{name}.npz", **record)
    print("wrote", name)


def _uvu_case(name, u, v, m_max, parity, parity_in2, normalization, path_normalization,
              shared, rows, seed, m_max_in2=None):
    torch = _torch()
    from ictc_o2_hp import ReferenceUvuTensorProduct
    tp = ReferenceUvuTensorProduct(u, v, m_max, parity=parity, parity_in2=parity_in2,
                                   m_max_in2=m_max_in2, normalization=normalization,
                                   path_normalization=path_normalization,
                                   shared_weights=shared).double()
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, tp.input1_dimension)).astype(np.float32)
    y = rng.standard_normal((rows, tp.input2_dimension)).astype(np.float32)
    wshape = (tp.weight_numel,) if shared else (rows, tp.weight_numel)
    w = (rng.standard_normal(wshape) / np.sqrt(v)).astype(np.float32)
    g = rng.standard_normal((rows, tp.representation_dimension)).astype(np.float32)
    xx, yy, ww = (torch.from_numpy(z).double().requires_grad_(True) for z in (x, y, w))
    out = tp(xx, yy, ww)
    dx, dy, dw = torch.autograd.grad(out, (xx, yy, ww), torch.from_numpy(g).double())
    np.savez_compressed(
        HERE / f"{name}.npz", u=u, v=v, m_max=m_max, m_max_in2=tp.m_max_in2, parity=parity,
        parity_in2=tp.parity_in2, normalization=normalization,
        path_normalization=path_normalization, shared=shared, x=x, y=y, w=w, g=g,
        out_f64=out.detach().numpy(), dx_f64=dx.numpy(), dy_f64=dy.numpy(), dw_f64=dw.numpy(),
        paths=np.array(tp.paths), coefficients=tp._coefficients.double().numpy())
    print("wrote", name)


def _radial_case(name, u, m_max, hidden, bias, rows, seed):
    torch = _torch()
    from ictc_o2_hp import ReferenceUvuTensorProduct, RadialUvuTensorProduct
    tp = ReferenceUvuTensorProduct(u, 1, m_max, parity="full", parity_in2="canonical",
                                   shared_weights=False)
    lin = torch.nn.Linear(hidden, tp.weight_numel, bias=bias)
    rng = np.random.default_rng(seed)
    alpha = (rng.standard_normal((tp.weight_numel, hidden)) / np.sqrt(hidden)).astype(np.float32)
    b = rng.standard_normal(tp.weight_numel).astype(np.float32) if bias else None
    x = rng.standard_normal((rows, tp.input1_dimension)).astype(np.float32)
    theta = rng.uniform(0, 2 * np.pi, rows)
    y = np.concatenate([np.ones((rows, 1))] + [
        np.stack([np.cos(m * theta), np.sin(m * theta)], -1) for m in range(1, m_max + 1)],
        axis=-1).astype(np.float32)
    h = rng.standard_normal((rows, hidden)).astype(np.float32)
    g = rng.standard_normal((rows, tp.representation_dimension)).astype(np.float32)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(alpha))
        if bias:
            lin.bias.copy_(torch.from_numpy(b))
    module = RadialUvuTensorProduct(tp, lin).double()
    xx, yy, hh = (torch.from_numpy(z).double().requires_grad_(True) for z in (x, y, h))
    out = module(xx, yy, hh)
    params = [module.radial_out.weight] + ([module.radial_out.bias] if bias else [])
    grads = torch.autograd.grad(out, (xx, yy, hh, *params), torch.from_numpy(g).double())
    record = dict(u=u, m_max=m_max, hidden=hidden, bias=bias, x=x, y=y, h=h, alpha=alpha, g=g,
                  out_f64=out.detach().numpy(), dx_f64=grads[0].numpy(),
                  dy_f64=grads[1].numpy(), dh_f64=grads[2].numpy(), da_f64=grads[3].numpy())
    if bias:
        record["b"] = b
        record["db_f64"] = grads[4].numpy()
    np.savez_compressed(HERE / f"{name}.npz", **record)
    print("wrote", name)


def _cg_tables(max_order=8):
    torch = _torch()
    from ictc_o2_hp import o2_math
    keys = [("scalar", 1), ("scalar", -1)] + [("freq", m) for m in range(1, max_order + 1)]
    names, values = [], []
    for k1 in keys:
        for k2 in keys:
            for k3 in o2_math.o2_valid_output_keys(k1, k2):
                if k3[0] == "freq" and k3[1] > max_order:
                    continue
                cg = o2_math.o2_cg_tensor(k1, k2, k3, dtype=torch.float64)
                names.append(f"{k1[0]}:{k1[1]}|{k2[0]}:{k2[1]}|{k3[0]}:{k3[1]}")
                padded = np.zeros((2, 2, 2))
                c = cg.numpy()
                padded[:c.shape[0], :c.shape[1], :c.shape[2]] = c
                values.append(padded)
    np.savez_compressed(HERE / "cg_tables.npz", names=np.array(names), cg=np.stack(values))
    print("wrote cg_tables")


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", default=os.environ.get("ICTC_REFERENCE_SRC"))
    parser.add_argument("--skip-large", action="store_true")
    args = parser.parse_args(argv)
    if args.reference_src:
        sys.path.insert(0, args.reference_src)
    f64 = [("f64", "float64")]
    both = [("f32", "float32"), ("f64", "float64")]

    def dt(pairs):
        torch = _torch()
        return [(tag, getattr(torch, name)) for tag, name in pairs]

    _cg_tables()
    # Config 1 of the benchmark recipe, whole N=4096 (rows kept: a sample + column sums).
    _tp_case("tp_c32_m2_canonical_cfg1", 32, 2, "canonical", "component", None, 0, "ones",
             dt(both), torch_rows=4096, keep_rows=list(range(16)) + [1000, 2047, 4095])
    _tp_case("tp_c32_m2_canonical_small", 32, 2, "canonical", "component", 40, 3, "random",
             dt(both))
    _tp_case("tp_c17_m3_full", 17, 3, "full", "component", 33, 5, "random", dt(f64))
    _tp_case("tp_c5_m4_canonical_norm", 5, 4, "canonical", "norm", 7, 7, "random", dt(f64))
    _tp_case("tp_c6_m5_full_norm", 6, 5, "full", "norm", 9, 8, "random", dt(f64))
    _tp_case("tp_c3_m0_full", 3, 0, "full", "component", 5, 9, "random", dt(f64))
    _tp_case("tp_c1_m1_canonical", 1, 1, "canonical", "component", 4, 10, "random", dt(f64))
    _tp_case("tp_c4_m8_full", 4, 8, "full", "component", 3, 11, "random", dt(f64))
    _tp_case("tp_c128_m6_full_small", 128, 6, "full", "component", 4, 12, "random", dt(both))
    if not args.skip_large:
        # Config 2 of the benchmark recipe: full N=65536, rows kept: a sample + sums.
        _tp_case("tp_c128_m6_full_cfg2", 128, 6, "full", "component", None, 0, "ones",
                 dt(both), torch_rows=65536, keep_rows=[0, 1, 2, 31337, 65535])
    _uvu_case("uvu_u16_v4_m3_full_shared", 16, 4, 3, "full", None, "component", "none", True,
              9, 21)
    _uvu_case("uvu_u8_v3_m2_full_perrow", 8, 3, 2, "full", None, "component", "none", False,
              5, 22)
    _uvu_case("uvu_u6_v1_m3_full_canonical2_perrow", 6, 1, 3, "full", "canonical", "component",
              "none", False, 7, 23)
    _uvu_case("uvu_u5_v2_m2_canonical_norm_path", 5, 2, 2, "canonical", None, "norm", "path",
              True, 6, 24)
    _uvu_case("uvu_u4_v3_m3_full_min2_element", 4, 3, 3, "full", "canonical", "component",
              "element", True, 5, 25, m_max_in2=2)
    _radial_case("radial_u8_m3_h16_bias", 8, 3, 16, True, 6, 31)
    _radial_case("radial_u4_m2_h5_nobias", 4, 2, 5, False, 5, 32)
    return 0


if __name__ == "__main__":
    sys.exit(main())
