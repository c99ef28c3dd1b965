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


def _chunks(rows, size):
    for start in range(0, rows, size):
        yield start, min(rows, start + size)


def _uvu_cfg4_shared(chunk=4096):
    """Config 4 with shared weights at its full 131,072 rows: the reference's float64
    CPU path over row chunks, the weight gradient summed across chunks (the
    validator's pattern, benchmarks/eqx/scripts/validate_math.py:54-74).  Kept:
    sampled rows, per-column sums of out / dx / dy and the whole dw."""
    torch = _torch()
    import recipes as R
    from ictc_o2_hp import ReferenceUvuTensorProduct
    c = R.CFG4
    tp = ReferenceUvuTensorProduct(c["u"], c["v"], c["m_max"], shared_weights=True).double()
    x, y, w, g = R.cfg4_shared_inputs()
    n = x.shape[0]
    keep = np.asarray(R.CFG4_SHARED_KEEP)
    wd = torch.from_numpy(w).double().requires_grad_(True)
    sums = {k: np.zeros(c["width2"] if k == "dy" else c["width1"]) for k in ("out", "dx", "dy")}
    rows = {k: np.zeros((len(keep), c["width2"] if k == "dy" else c["width1"]))
            for k in ("out", "dx", "dy")}
    dw = np.zeros(c["weight_numel"])
    for s, e in _chunks(n, chunk):
        xx = torch.from_numpy(x[s:e]).double().requires_grad_(True)
        yy = torch.from_numpy(y[s:e]).double().requires_grad_(True)
        out = tp(xx, yy, wd)
        gx, gy, gw = torch.autograd.grad(out, (xx, yy, wd), torch.from_numpy(g[s:e]).double())
        dw += gw.numpy()
        for key, value in (("out", out.detach()), ("dx", gx), ("dy", gy)):
            v = value.numpy()
            sums[key] += v.sum(axis=0)
            sel = (keep >= s) & (keep < e)
            rows[key][sel] = v[keep[sel] - s]
        print(f"  cfg4 shared rows {e}/{n}", flush=True)
    record = {f"{k}_f64_rows": rows[k] for k in rows}
    record.update({f"{k}_f64_sum": sums[k] for k in sums})
    record.update(dw_f64=dw, keep_rows=keep, rows=n, seed=R.CFG4_SHARED_SEED)
    np.savez_compressed(HERE / "full_uvu_cfg4_shared.npz", **record)
    print("wrote full_uvu_cfg4_shared")


def _uvu_cfg4_perrow():
    """Config 4 with per-row weights: the reference's float64 values of the sampled
    rows (each row's inputs from its own seeded stream, recipes.cfg4_perrow_row)."""
    torch = _torch()
    import recipes as R
    from ictc_o2_hp import ReferenceUvuTensorProduct
    c = R.CFG4
    tp = ReferenceUvuTensorProduct(c["u"], c["v"], c["m_max"], shared_weights=False).double()
    parts = [R.cfg4_perrow_row(r) for r in R.CFG4_PERROW_KEEP]
    x, y, w, g = (torch.from_numpy(np.stack([p[i] for p in parts])).double() for i in range(4))
    x.requires_grad_(True), y.requires_grad_(True), w.requires_grad_(True)
    out = tp(x, y, w)
    dx, dy, dw = torch.autograd.grad(out, (x, y, w), g)
    # a row of dw is as large as a row of weights (606,208 values): keep a fixed
    # strided subset of its entries (every row is also checked in full on the GPU
    # against the float64 formula)
    cols = np.asarray(R.CFG4_PERROW_DW_COLUMNS)
    np.savez_compressed(
        HERE / "full_uvu_cfg4_perrow_rows.npz", keep_rows=np.asarray(R.CFG4_PERROW_KEEP),
        rows=R.CFG4_PERROW_ROWS, seed=R.CFG4_PERROW_SEED, out_f64=out.detach().numpy(),
        dx_f64=dx.numpy(), dy_f64=dy.numpy(), dw_columns=cols, dw_f64=dw.numpy()[:, cols])
    print("wrote full_uvu_cfg4_perrow_rows")


def _radial_cfg5(chunk=8192):
    """Config 5 at its full 1,048,576 edges through the reference's composition
    ``tp(left, angular, radial_out(hidden))`` (radial_uvu.py:50-52) in float64 on the
    CPU, over edge chunks with the affine-layer gradients summed across chunks
    (the accumulation of radial_streamed.py:126-138).  Kept: sampled edges,
    per-column sums of out / dx / dangular / dhidden, the whole dalpha and dbias."""
    torch = _torch()
    import recipes as R
    from ictc_o2_hp import RadialUvuTensorProduct, ReferenceUvuTensorProduct
    c = R.CFG5
    d = R.cfg5_inputs()
    tp = ReferenceUvuTensorProduct(c["u"], 1, c["m_max"], parity="full",
                                   parity_in2="canonical", shared_weights=False)
    lin = torch.nn.Linear(c["hidden"], c["weight_numel"], bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(d["alpha"]))
        lin.bias.copy_(torch.from_numpy(d["bias"]))
    module = RadialUvuTensorProduct(tp, lin).double()
    params = (module.radial_out.weight, module.radial_out.bias)
    n = d["src"].shape[0]
    keep = np.asarray(R.CFG5_KEEP)
    widths = {"out": c["width1"], "dx": c["width1"], "dy": c["width2"], "dh": c["hidden"]}
    sums = {k: np.zeros(v) for k, v in widths.items()}
    rows = {k: np.zeros((len(keep), v)) for k, v in widths.items()}
    da = np.zeros((c["weight_numel"], c["hidden"]))
    db = np.zeros(c["weight_numel"])
    for s, e in _chunks(n, chunk):
        xx = torch.from_numpy(d["nodes"][d["src"][s:e]]).double().requires_grad_(True)
        yy = torch.from_numpy(d["angular"][s:e]).double().requires_grad_(True)
        hh = torch.from_numpy(d["hidden"][s:e]).double().requires_grad_(True)
        out = module(xx, yy, hh)
        gx, gy, gh, ga, gb = torch.autograd.grad(
            out, (xx, yy, hh, *params), torch.from_numpy(d["g"][s:e]).double())
        da += ga.numpy()
        db += gb.numpy()
        for key, value in (("out", out.detach()), ("dx", gx), ("dy", gy), ("dh", gh)):
            v = value.numpy()
            sums[key] += v.sum(axis=0)
            sel = (keep >= s) & (keep < e)
            rows[key][sel] = v[keep[sel] - s]
        if (e // chunk) % 16 == 0 or e == n:
            print(f"  cfg5 edges {e}/{n}", flush=True)
    record = {f"{k}_f64_rows": rows[k] for k in rows}
    record.update({f"{k}_f64_sum": sums[k] for k in sums})
    record.update(da_f64=da, db_f64=db, keep_rows=keep, edges=n, seed=R.CFG5_SEED)
    np.savez_compressed(HERE / "full_radial_cfg5.npz", **record)
    print("wrote full_radial_cfg5")


def _second_order(create, inputs, first_roles, extra=()):
    """Second derivatives of S = sum_r <d(out . g)/d role_r, h_r> with respect to every
    operand and the cotangent g, by the reference's own autograd (create_graph)."""
    torch = _torch()
    out = create(*inputs)
    g, hs = extra[0], extra[1:]
    firsts = torch.autograd.grad(out, first_roles, g, create_graph=True)
    total = sum((f * h).sum() for f, h in zip(firsts, hs))
    return torch.autograd.grad(total, (*first_roles, g))


def _tp_second_case(name, channels, m_max, parity, normalization, rows, seed):
    """TensorProduct second derivatives (reference CPU autograd over fast_o2.py:80-149,
    the map whose double backward triton_o2.py:1041-1069 recomputes)."""
    torch = _torch()
    from ictc_o2_hp import TensorProduct
    tp = TensorProduct(channels, m_max, parity=parity, normalization=normalization)
    tp = tp.to(torch.float64)
    tp.internal_compute_dtype = torch.float64
    width = tp.representation_dimension
    rng = np.random.default_rng(seed)
    arrays = {k: rng.standard_normal((rows, width)).astype(np.float32)
              for k in ("x", "y", "g", "hx", "hy")}
    arrays["w"] = rng.standard_normal(tp.weight.numel()).astype(np.float32)
    arrays["hw"] = rng.standard_normal(tp.weight.numel()).astype(np.float32)
    t = {k: torch.from_numpy(v).double() for k, v in arrays.items()}
    with torch.no_grad():
        tp.weight.copy_(t["w"])
    x, y, g = (t[k].requires_grad_(True) for k in ("x", "y", "g"))
    sx, sy, sw, sg = _second_order(lambda a, b: tp(a, b), (x, y), (x, y, tp.weight),
                                   (g, t["hx"], t["hy"], t["hw"]))
    np.savez_compressed(HERE / f"{name}.npz", channels=channels, m_max=m_max, parity=parity,
                        normalization=normalization, **arrays, sx_f64=sx.numpy(),
                        sy_f64=sy.numpy(), sw_f64=sw.numpy(), sg_f64=sg.numpy())
    print("wrote", name)


def _uvu_second_case(name, u, v, m_max, shared, rows, seed):
    torch = _torch()
    from ictc_o2_hp import ReferenceUvuTensorProduct
    tp = ReferenceUvuTensorProduct(u, v, m_max, shared_weights=shared,
                                   internal_weights=False).double()
    rng = np.random.default_rng(seed)
    wshape = (tp.weight_numel,) if shared else (rows, tp.weight_numel)
    arrays = {"x": rng.standard_normal((rows, tp.input1_dimension)),
              "y": rng.standard_normal((rows, tp.input2_dimension)),
              "w": rng.standard_normal(wshape) / np.sqrt(v),
              "g": rng.standard_normal((rows, tp.representation_dimension)),
              "hx": rng.standard_normal((rows, tp.input1_dimension)),
              "hy": rng.standard_normal((rows, tp.input2_dimension)),
              "hw": rng.standard_normal(wshape)}
    arrays = {k: a.astype(np.float32) for k, a in arrays.items()}
    t = {k: torch.from_numpy(a).double() for k, a in arrays.items()}
    x, y, w, g = (t[k].requires_grad_(True) for k in ("x", "y", "w", "g"))
    sx, sy, sw, sg = _second_order(lambda a, b, c: tp(a, b, c), (x, y, w), (x, y, w),
                                   (g, t["hx"], t["hy"], t["hw"]))
    np.savez_compressed(HERE / f"{name}.npz", u=u, v=v, m_max=m_max, shared=shared, **arrays,
                        sx_f64=sx.numpy(), sy_f64=sy.numpy(), sw_f64=sw.numpy(),
                        sg_f64=sg.numpy())
    print("wrote", name)


def _radial_second_case(name, u, m_max, hidden, bias, rows, seed):
    """Radial second derivatives through the reference composition (the map whose
    double backward radial_streamed.py:173-207 recomputes)."""
    torch = _torch()
    from ictc_o2_hp import RadialUvuTensorProduct, ReferenceUvuTensorProduct
    tp = ReferenceUvuTensorProduct(u, 1, m_max, parity="full", parity_in2="canonical",
                                   shared_weights=False)
    lin = torch.nn.Linear(hidden, tp.weight_numel, bias=bias)
    rng = np.random.default_rng(seed)
    arrays = {"x": rng.standard_normal((rows, tp.input1_dimension)),
              "y": rng.standard_normal((rows, tp.input2_dimension)),
              "h": rng.standard_normal((rows, hidden)),
              "alpha": rng.standard_normal((tp.weight_numel, hidden)) / np.sqrt(hidden),
              "g": rng.standard_normal((rows, tp.representation_dimension)),
              "hx": rng.standard_normal((rows, tp.input1_dimension)),
              "hy": rng.standard_normal((rows, tp.input2_dimension)),
              "hh": rng.standard_normal((rows, hidden)),
              "ha": rng.standard_normal((tp.weight_numel, hidden))}
    if bias:
        arrays["b"] = rng.standard_normal(tp.weight_numel)
        arrays["hb"] = rng.standard_normal(tp.weight_numel)
    arrays = {k: a.astype(np.float32) for k, a in arrays.items()}
    t = {k: torch.from_numpy(a).double() for k, a in arrays.items()}
    with torch.no_grad():
        lin.weight.copy_(t["alpha"].float())
        if bias:
            lin.bias.copy_(t["b"].float())
    module = RadialUvuTensorProduct(tp, lin).double()
    x, y, h, g = (t[k].requires_grad_(True) for k in ("x", "y", "h", "g"))
    params = (module.radial_out.weight,) + ((module.radial_out.bias,) if bias else ())
    hs = (t["hx"], t["hy"], t["hh"], t["ha"]) + ((t["hb"],) if bias else ())
    result = _second_order(lambda a, b, c: module(a, b, c), (x, y, h), (x, y, h, *params),
                           (g, *hs))
    keys = ["sx", "sy", "sh", "sa"] + (["sb"] if bias else []) + ["sg"]
    np.savez_compressed(HERE / f"{name}.npz", u=u, m_max=m_max, hidden=hidden, bias=bias,
                        **arrays, **{f"{k}_f64": r.numpy() for k, r in zip(keys, result)})
    print("wrote", name)


def _layout_case(name, cls_name, channels, m_max, parity, normalization, rows, seed):
    """ComponentMajorTensorProduct / TupleTensorProduct forward and VJP by the
    reference's own classes (api.py:32-49) in float64 on the CPU.  Tuple inputs and
    outputs are stored as the flat concatenation of their blocks in block order."""
    torch = _torch()
    import ictc_o2_hp
    cls = getattr(ictc_o2_hp, cls_name)
    tp = cls(channels, m_max, parity=parity, normalization=normalization).to(torch.float64)
    tp.internal_compute_dtype = torch.float64
    width = tp.representation_dimension
    rng = np.random.default_rng(seed)
    arrays = {k: rng.standard_normal((rows, width)).astype(np.float32) for k in ("x", "y", "g")}
    arrays["w"] = (0.5 * rng.standard_normal(tp.weight.numel())).astype(np.float32)
    with torch.no_grad():
        tp.weight.copy_(torch.from_numpy(arrays["w"]).double())
    x, y, g = (torch.from_numpy(arrays[k]).double() for k in ("x", "y", "g"))
    x.requires_grad_(True), y.requires_grad_(True)
    if cls_name == "TupleTensorProduct":
        def split(value):
            parts, cursor = [], 0
            for block in tp.blocks:
                width_b = block.multiplicity * block.irrep_dimension
                parts.append(value[:, cursor:cursor + width_b].reshape(
                    rows, block.multiplicity, block.irrep_dimension))
                cursor += width_b
            return tuple(parts)
        out = torch.cat([v.reshape(rows, -1) for v in tp(split(x), split(y))], dim=-1)
    else:
        out = tp(x, y)
    dx, dy, dw = torch.autograd.grad(out, (x, y, tp.weight), g)
    np.savez_compressed(HERE / f"{name}.npz", cls=cls_name, channels=channels, m_max=m_max,
                        parity=parity, normalization=normalization, **arrays,
                        out_f64=out.detach().numpy(), dx_f64=dx.numpy(), dy_f64=dy.numpy(),
                        dw_f64=dw.numpy())
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
    parser.add_argument("--only", nargs="*", default=None,
                        help="groups to write: base, full, second, layout (default: all)")
    args = parser.parse_args(argv)
    if args.reference_src:
        sys.path.insert(0, args.reference_src)
    sys.path.insert(0, str(HERE))
    groups = set(args.only or ("base", "full", "second", "layout"))
    if "second" in groups:
        _tp_second_case("second_tp_c6_m3_full", 6, 3, "full", "component", 5, 41)
        _tp_second_case("second_tp_c5_m2_canonical_norm", 5, 2, "canonical", "norm", 4, 42)
        _tp_second_case("second_tp_c3_m6_full", 3, 6, "full", "component", 3, 43)
        _uvu_second_case("second_uvu_u6_v3_m2_shared", 6, 3, 2, True, 5, 44)
        _uvu_second_case("second_uvu_u5_v2_m3_perrow", 5, 2, 3, False, 4, 45)
        _radial_second_case("second_radial_u4_m2_h5_bias", 4, 2, 5, True, 5, 46)
        _radial_second_case("second_radial_u6_m3_h4_nobias", 6, 3, 4, False, 4, 47)
    if "layout" in groups:
        _layout_case("layout_cm_c7_m3_full", "ComponentMajorTensorProduct", 7, 3, "full",
                     "component", 6, 51)
        _layout_case("layout_cm_c5_m4_canonical_norm", "ComponentMajorTensorProduct", 5, 4,
                     "canonical", "norm", 5, 52)
        _layout_case("layout_tuple_c6_m2_full", "TupleTensorProduct", 6, 2, "full",
                     "component", 4, 53)
        _layout_case("layout_tuple_c4_m5_canonical", "TupleTensorProduct", 4, 5, "canonical",
                     "component", 3, 54)
    if "full" in groups:
        _uvu_cfg4_perrow()
        _uvu_cfg4_shared()
        _radial_cfg5()
    if "base" not in groups:
        return 0
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
