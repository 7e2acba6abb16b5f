"""Per-shape kernel selection, retrained on B200 (counterpart of tilec/tune.py).

    python -m tilec_b200.tune bench  [--shapes N] [--csv PATH]   sweep shapes x configs, append CSV
    python -m tilec_b200.tune train  [--csv PATH] [--out PATH]   fit the JSON selection table
    python -m tilec_b200.tune run    --shape M,K,N [--variant V] [--split S] [--reps R]

``bench`` mirrors tilec/tune.py:68-87: seeded shapes, every candidate config of
``ext.kernel_configs`` timed, resumable (shapes already in the CSV are skipped).  Timing is
CUDA events around back-to-back launches after warm-up (tilec/tune.py:35-51 used
perf_counter + synchronize and a median of 5), with the same early abort for configs far
slower than the best so far.  The shape sampler follows tilec/tune.py:54-65 but spans
[1, 8192] per dimension (benchmark config 4) and includes M = 1 and N <= 64 cases.

``train`` mirrors tilec/tune.py:99-132: a held-out 20% of shapes measures the geo-mean
"x of best" of the fitted selector against the library's built-in rules
(tilec/tune.py:125-128), then the table is refit on all shapes and written as JSON (the
reference pickles a sklearn model, tune.py:131-132; a JSON table loads without running
code).  The table maps log2-size boxes to (variant, split_k); see tilec_b200/select.py.

``run`` launches one shape a few times (for profiler captures).
"""
import argparse
import csv
import json
import math
import os
import random
import sys

FIELDS = ["device", "M", "K", "N", "variant", "split_k", "ms"]
DEFAULT_CSV = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mm_bench_b200.csv")


def shapes(n=64, seed=4):
    """Seeded log-uniform (M, K, N) over [1, 8192]^3; first M = 1, second N <= 64."""
    rng = random.Random(seed)
    out, seen = [], set()
    while len(out) < n:
        m, k, nn = (max(1, round(2 ** rng.uniform(0, 13))) for _ in range(3))
        if len(out) == 0:
            m = 1
        elif len(out) == 1:
            nn = min(nn, 64)
        if (m, k, nn) in seen:
            continue
        seen.add((m, k, nn))
        out.append((m, k, nn))
    return out


def time_ms(fn, best=None, reps=None):
    """Mean CUDA-event time of fn() per call; aborts early when far slower than `best`."""
    import torch
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    fn()
    e.record()
    torch.cuda.synchronize()
    first = s.elapsed_time(e)
    if best is not None and first > 2 * best:
        return first
    if reps is None:
        reps = max(3, min(200, int(20.0 / max(first, 1e-3))))
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def load(path=DEFAULT_CSV):
    with open(path) as f:
        rows = []
        for r in csv.DictReader(f):
            rows.append({"device": r["device"], "M": int(r["M"]), "K": int(r["K"]), "N": int(r["N"]),
                         "variant": r["variant"], "split_k": int(r["split_k"]), "ms": float(r["ms"])})
        return rows


def bench(n=64, path=DEFAULT_CSV, seed=4):
    import torch
    from . import ext
    dev = torch.cuda.get_device_name()
    done = {(r["M"], r["K"], r["N"]) for r in load(path)} if os.path.exists(path) else set()
    new = not os.path.exists(path)
    with open(path, "a", newline="") as f:
        w = csv.writer(f)
        if new:
            w.writerow(FIELDS)
        for i, (m, k, nn) in enumerate(shapes(n, seed)):
            if (m, k, nn) in done:
                continue
            g = torch.Generator(device="cuda").manual_seed(i)
            a = torch.randn(m, k, device="cuda", generator=g)
            b = torch.randn(k, nn, device="cuda", generator=g)
            c = torch.empty(m, nn, device="cuda")
            best = None
            # Built-in rules (no table) and each variant family with the library's own split.
            from . import select
            select.install([])
            auto = lambda: ext._matrix_mul(a, b, variant="auto", out=c)  # noqa: E731
            ms_auto = time_ms(auto)
            cands = [("simt", 0), ("splitk", 0), ("3xtf32", 0), ("tf32", 0)] + ext.kernel_configs(m, k, nn)
            out_rows = []
            for v, s in cands:
                # Family rows (the library's own split) feed the fit, so they are always
                # measured in full; explicit splits may stop early when far behind.
                ms = time_ms(lambda: ext._matrix_mul(a, b, variant=v, split_k=s, out=c), None if s == 0 else best)
                best = ms if best is None else min(best, ms)
                out_rows.append([dev, m, k, nn, v, s, f"{ms:.6f}"])
            # The built-in rule is timed before and after the families and keeps the faster:
            # the first calls on fresh operands read a few microseconds slow, which at the
            # launch floor would otherwise look like a loss of the rule.
            ms_auto = min(ms_auto, time_ms(auto))
            w.writerow([dev, m, k, nn, "builtin", 0, f"{ms_auto:.6f}"])
            w.writerows(out_rows)
            f.flush()
            print(f"{i + 1}/{n}  {m}x{k} @ {k}x{nn}  best {best:.4f} ms", flush=True)


def _box(m, k, n):
    lg = lambda v: max(int(v), 1).bit_length() - 1  # noqa: E731
    return lg(m), lg(n), lg(k)


# AUTO must keep fp32-class accuracy (relFrob <= 1e-5), so plain TF32 is measured but never chosen.
FP32_CLASS = ("simt", "splitk", "3xtf32")
GRID_EDGES = (0, 2, 4, 6, 8, 10, 12, 64)   # log2-size bins (2 octaves wide; the last is open)


def _family_rows(rows):
    """Rows timed with the library's own split choice (split_k == 0), fp32-class only."""
    return [r for r in rows if r["variant"] in FP32_CLASS and r["split_k"] == 0]


def _best_family(rs):
    return min(rs, key=lambda r: r["ms"])["variant"]


def fit(rows, k_nn=3, margin=1.10):
    """Selection rows over a coarse log2 grid, only where the measurements beat the
    library's built-in rule: a cell gets the variant family that is fastest for the
    majority of the k_nn measured shapes nearest to its centre (log2 space), provided
    that family is at least `margin` times faster than the built-in choice on those
    shapes (geometric mean).  Other cells get no row, so AUTO keeps its built-in rule
    there.  The split count is left to the library (split_k = 0)."""
    by_shape = {}
    for r in rows:
        by_shape.setdefault((r["M"], r["K"], r["N"]), []).append(r)
    pts = []
    for (m, k, n), rs in by_shape.items():
        fam = {r["variant"]: r["ms"] for r in rs if r["variant"] in FP32_CLASS and r["split_k"] == 0}
        builtin = next((r["ms"] for r in rs if r["variant"] == "builtin"), None)
        if fam and builtin is not None:
            pts.append(((math.log2(max(m, 1)), math.log2(max(n, 1)), math.log2(max(k, 1))), fam, builtin))
    if not pts:
        return []
    table = []
    e = GRID_EDGES
    for i in range(len(e) - 1):
        for j in range(len(e) - 1):
            for l in range(len(e) - 1):
                c = tuple(min(e[x] + 1.0, 13.0) for x in (i, j, l))
                near = sorted(pts, key=lambda p: sum((p[0][d] - c[d]) ** 2 for d in range(3)))[:k_nn]
                votes = {}
                for _, fam, _ in near:
                    best = min(fam, key=fam.get)
                    votes[best] = votes.get(best, 0) + 1
                v, count = max(votes.items(), key=lambda kv: (kv[1], kv[0] == "3xtf32"))
                if count <= len(near) // 2 or any(v not in fam for _, fam, _ in near):
                    continue
                gain = math.exp(sum(math.log(b / fam[v]) for _, fam, b in near) / len(near))
                if gain >= margin:
                    table.append([e[i], e[i + 1], e[j], e[j + 1], e[l], e[l + 1], v, 0])
    return table


def train(path=DEFAULT_CSV, out=None, test_frac=0.2, seed=0):
    from . import select
    rows = load(path)
    fam = _family_rows(rows)
    keys = sorted({(r["M"], r["K"], r["N"]) for r in fam})
    random.Random(seed).shuffle(keys)
    test = set(keys[: int(len(keys) * test_frac)])
    table = fit([r for r in rows if (r["M"], r["K"], r["N"]) not in test])
    by_shape = {}
    for r in rows:
        by_shape.setdefault((r["M"], r["K"], r["N"]), []).append(r)
    ratio_sel, ratio_default = [], []
    for key in test:
        rs = by_shape[key]
        best = min(r["ms"] for r in rs if r["variant"] in FP32_CLASS)
        pick = select.lookup([t[:6] + [_variant_code(t[6]), t[7]] for t in table], *_mnk(key))
        default = next(r for r in rs if r["variant"] == "builtin")
        chosen = default if pick is None else next(r for r in rs if r["variant"] == pick[0] and r["split_k"] == 0)
        ratio_sel.append(chosen["ms"] / best)
        ratio_default.append(default["ms"] / best)
    gm = lambda v: math.exp(sum(math.log(a) for a in v) / max(len(v), 1))  # noqa: E731
    cv = cross_validate(rows)
    print(f"5-fold cross-validation over all {len(keys)} shapes: selector {cv['selector_x_of_best']:.3f}x of best "
          f"(worst {cv['selector_worst']:.2f}x), built-in rules {cv['builtin_x_of_best']:.3f}x "
          f"(worst {cv['builtin_worst']:.2f}x)")
    print(f"held-out shapes: {len(test)}")
    print(f"selector: {gm(ratio_sel):.3f}x of best (geo mean), worst {max(ratio_sel, default=1):.2f}x")
    print(f"default : {gm(ratio_default):.3f}x of best (geo mean), worst {max(ratio_default, default=1):.2f}x")
    table = fit(rows)
    # A table ships only if it beats the built-in rules under cross-validation; otherwise its
    # rows fit measurement noise (launch-floor shapes differ by a few microseconds from run
    # to run) and AUTO stays the built-in rule.
    kept = cv["selector_x_of_best"] < cv["builtin_x_of_best"]
    if not kept and table:
        print(f"cross-validation: the fitted table ({len(table)} rows) does not beat the built-in rules; "
              "writing an empty table")
        table = []
    doc = {"device": rows[0]["device"] if rows else "", "source": os.path.basename(path),
           "shapes": len(keys), "grid_log2_edges": list(GRID_EDGES), "rows": table,
           "fitted_table_kept": kept,
           "heldout": {"shapes": len(test), "selector_x_of_best": round(gm(ratio_sel), 4),
                       "builtin_x_of_best": round(gm(ratio_default), 4),
                       "selector_worst": round(max(ratio_sel, default=1), 3),
                       "builtin_worst": round(max(ratio_default, default=1), 3)},
           "cross_validation": cv}
    out = out or select.TABLE_PATH
    with open(out, "w") as f:
        json.dump(doc, f, indent=1)
    print("wrote", out)
    return doc


def _choice_ms(rs, table):
    """Time of what AUTO runs for one measured shape under `table` (the built-in rule's
    time when no row matches)."""
    from . import select
    m, k, n = rs[0]["M"], rs[0]["K"], rs[0]["N"]
    pick = select.lookup([t[:6] + [_variant_code(t[6]), t[7]] for t in table], m, n, k)
    default = next(r for r in rs if r["variant"] == "builtin")
    if pick is None:
        return default["ms"]
    return next(r for r in rs if r["variant"] == pick[0] and r["split_k"] == 0)["ms"]


def cross_validate(rows, folds=5, seeds=(0, 1, 2)):
    """k-fold estimate (averaged over shuffles) of the fitted selector and of the built-in
    rules, as geometric-mean and worst "x of best" over every measured shape."""
    by_shape = {}
    for r in rows:
        by_shape.setdefault((r["M"], r["K"], r["N"]), []).append(r)
    keys0 = sorted(k for k, rs in by_shape.items() if any(r["variant"] == "builtin" for r in rs))
    sel, dft = [], []
    for seed in seeds:
        keys = list(keys0)
        random.Random(seed).shuffle(keys)
        for f in range(folds):
            test = set(keys[f::folds])
            table = fit([r for r in rows if (r["M"], r["K"], r["N"]) not in test])
            for key in test:
                rs = by_shape[key]
                best = min(r["ms"] for r in rs if r["variant"] in FP32_CLASS)
                sel.append(_choice_ms(rs, table) / best)
                dft.append(next(r for r in rs if r["variant"] == "builtin")["ms"] / best)
    gm = lambda v: math.exp(sum(math.log(a) for a in v) / max(len(v), 1))  # noqa: E731
    return {"folds": folds, "shuffles": len(seeds), "selector_x_of_best": round(gm(sel), 4),
            "builtin_x_of_best": round(gm(dft), 4), "selector_worst": round(max(sel, default=1), 3),
            "builtin_worst": round(max(dft, default=1), 3)}


def _variant_code(v):
    from . import _native
    return _native.VARIANTS[v]


def _mnk(key):
    m, k, n = key
    return m, n, k


def pick(M, K, N):
    """(variant, split_k) that matrix_mul launches for an [M,K] x [K,N] product."""
    import torch
    from . import ext
    a = torch.empty(M, K, device="cuda")
    b = torch.empty(K, N, device="cuda")
    return ext.kernel_plan(a, b)


def run(shape, variant="auto", split=0, reps=3, seed=0, stream_k=False, batch=0, tile_m=None):
    """One warm-up call, then `reps` back-to-back calls of one product timed with CUDA
    events (for profilers and A/B runs); prints the plan that ran and the mean time per call.
    batch > 0: one matrix_mul_ex call over `batch` products of the shape per launch."""
    import torch
    from . import ext
    m, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(seed)
    lead = (batch,) if batch > 0 else ()
    a = torch.randn(*lead, m, k, device="cuda", generator=g)
    b = torch.randn(*lead, k, n, device="cuda", generator=g)
    c = torch.empty(*lead, m, n, device="cuda")

    def call():
        if batch > 0:
            ext.matrix_mul_ex(a, b, out=c, variant=variant, split_k=split, stream_k=stream_k, tile_m=tile_m)
        else:
            ext._matrix_mul(a, b, variant=variant, split_k=split, out=c, stream_k=stream_k, tile_m=tile_m)
    call()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        call()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / max(reps, 1)
    a0, b0 = (a[0], b[0]) if batch > 0 else (a, b)
    plan = ext.kernel_plan(a0, b0, variant=variant, split_k=split, stream_k=stream_k, detail=True, tile_m=tile_m)
    flops = 2.0 * m * n * k * max(batch, 1)
    print(json.dumps({"shape": [m, k, n], "batch": batch, "plan": plan, "reps": reps, "ms_per_call": round(ms, 4),
                      "tflops": round(flops / ms / 1e9, 2)}))


def main(argv=None):
    p = argparse.ArgumentParser(prog="python -m tilec_b200.tune")
    sub = p.add_subparsers(dest="cmd", required=True)
    pb = sub.add_parser("bench")
    pb.add_argument("--shapes", type=int, default=64)
    pb.add_argument("--seed", type=int, default=4)
    pb.add_argument("--csv", default=DEFAULT_CSV)
    pt = sub.add_parser("train")
    pt.add_argument("--csv", default=DEFAULT_CSV)
    pt.add_argument("--out", default=None)
    pr = sub.add_parser("run")
    pr.add_argument("--shape", required=True)
    pr.add_argument("--variant", default="auto")
    pr.add_argument("--split", type=int, default=0)
    pr.add_argument("--reps", type=int, default=3)
    pr.add_argument("--stream-k", action="store_true", help="ask for the pair kernel's stream-K form")
    pr.add_argument("--batch", type=int, default=0, help="run a batch of this many products per launch")
    pr.add_argument("--tile-m", type=int, default=None, choices=[64, 128],
                    help="rows per tile of the 1-CTA tensor-core kernel")
    args = p.parse_args(argv)
    if args.cmd == "bench":
        bench(args.shapes, args.csv, args.seed)
    elif args.cmd == "train":
        train(args.csv, args.out)
    else:
        run(tuple(int(x) for x in args.shape.split(",")), args.variant, args.split, args.reps,
            stream_k=args.stream_k, batch=args.batch, tile_m=args.tile_m)


if __name__ == "__main__":
    sys.exit(main())
