"""Tuning cache and autotuner for the tensor-core GEMM (the reference's
lib/Autotune + lib/Runtime/KernelCache, re-done around tcgen05 tile shapes).

* `ConfigSpace` enumerates tcgen05 GEMM configs (tile width block_n and pipeline
  depth shared_memory_stages; block_m, block_k, warps, vector width and TMEM
  accumulator count are fixed by the kernel) and prunes those that do not fit
  shared memory (227 KB per CTA) or TMEM (512 columns), like ConfigSpace's prune
  rules (lib/Autotune/ConfigSpace.cpp:44-142). Only configs with a compiled
  variant survive.
* `autotune` times every surviving config on the GPU, gates each on
  correctness (bit-identical to the default variant -- the K reduction order does
  not depend on the tile width or depth -- and cosine / max_rel_err / PCC
  against an fp32 torch reference of the same product), and picks the fastest
  validated one (Benchmark.cpp:31-52 semantics: an unvalidated config is never
  selected).
* `load` / `save` / `validate` read and write cache files in the reference's
  format (tuning/schema.json, version 1; restated in tuning_schema.json here).
  The C runtime (`pkb200_tuning_load`) parses the same files with the same rules.
"""
from __future__ import annotations

import ctypes
import json
import os

SCHEMA_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tuning_schema.json")
CONFIG_FIELDS = ("block_m", "block_n", "block_k", "num_warps", "vector_width", "unroll",
                 "shared_memory_stages")
SMEM_LIMIT = 232448          # bytes per CTA on sm_100
TMEM_COLUMNS = 512
# (block_m, block_n, stages) with a compiled kernel; block_m 256 is the CTA-pair
# (cta_group::2) kernel: two SMs share a 256 x block_n tile, each staging half of
# A and half of B
COMPILED = {(128, 256, 4), (128, 256, 3), (128, 128, 4), (128, 128, 6), (256, 256, 6)}
DEFAULT = dict(block_m=128, block_n=256, block_k=64, num_warps=10, vector_width=8, unroll=2,
               shared_memory_stages=4)


class SchemaError(ValueError):
    pass


# ------------------------------------------------------------ config space --
class ConfigSpace:
    """tcgen05 GEMM configs: CTAs per tile (block_m 128: one SM; 256: a CTA
    pair on two SMs, cta_group::2) x block_n x stages over the kernel's fixed
    axes."""
    block_m = (128, 256)
    block_n = (64, 128, 256)
    stages = (2, 3, 4, 5, 6, 7, 8)

    @staticmethod
    def smem_bytes(c):
        # per CTA: a pair tile splits A by rows and B by columns between its CTAs
        ctas = c["block_m"] // 128
        stage = (c["block_m"] // ctas) * c["block_k"] * 2 + c["block_k"] * (c["block_n"] // ctas) * 2
        return c["shared_memory_stages"] * stage + 1024 + 512  # + alignment, barriers/tile ring

    @classmethod
    def prune_reason(cls, c):
        if cls.smem_bytes(c) > SMEM_LIMIT:
            return "shared memory"
        if c["unroll"] * c["block_n"] > TMEM_COLUMNS:
            return "tmem columns"
        if (c["block_m"], c["block_n"], c["shared_memory_stages"]) not in COMPILED:
            return "no compiled variant"
        return None

    @classmethod
    def enumerate(cls, limit=None):
        out = []
        for bm in cls.block_m:
            for bn in cls.block_n:
                for st in cls.stages:
                    c = dict(DEFAULT, block_m=bm, block_n=bn, shared_memory_stages=st)
                    if cls.prune_reason(c) is None:
                        out.append(c)
        return out[:limit] if limit else out


# ----------------------------------------------------------------- schema --
def _check_keys(obj, keys, where):
    if not isinstance(obj, dict):
        raise SchemaError(f"{where}: expected an object")
    extra = set(obj) - set(keys)
    if extra:
        raise SchemaError(f"{where}: unknown field '{sorted(extra)[0]}'")
    missing = [k for k in keys if k not in obj]
    if missing:
        raise SchemaError(f"{where}: missing field '{missing[0]}'")


def _is_int(v):
    return isinstance(v, int) and not isinstance(v, bool)


def _is_num(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def validate(doc):
    """Raise SchemaError unless `doc` is a valid version-1 cache document."""
    _check_keys(doc, ("version", "entries"), "cache")
    if not _is_int(doc["version"]) or doc["version"] != 1:
        raise SchemaError(f"cache.version: unsupported version {doc['version']!r} (expected 1)")
    if not isinstance(doc["entries"], list):
        raise SchemaError("cache.entries: expected an array")
    for i, e in enumerate(doc["entries"]):
        w = f"entries[{i}]"
        _check_keys(e, ("gpu", "op", "shape", "best", "scored_by", "time_ms", "validated",
                        "correctness"), w)
        for k in ("gpu", "op"):
            if not isinstance(e[k], str):
                raise SchemaError(f"{w}.{k}: expected a string")
        _check_keys(e["shape"], ("M", "N", "K", "dtype"), w + ".shape")
        for k in ("M", "N", "K"):
            if not _is_int(e["shape"][k]):
                raise SchemaError(f"{w}.shape.{k}: expected an integer")
        if not isinstance(e["shape"]["dtype"], str):
            raise SchemaError(f"{w}.shape.dtype: expected a string")
        _check_keys(e["best"], CONFIG_FIELDS, w + ".best")
        for k in CONFIG_FIELDS:
            if not _is_int(e["best"][k]):
                raise SchemaError(f"{w}.best.{k}: expected an integer")
        if e["scored_by"] not in ("measure", "compile_time_model"):
            raise SchemaError(f"{w}.scored_by: must be measure or compile_time_model")
        if e["time_ms"] is not None and not _is_num(e["time_ms"]):
            raise SchemaError(f"{w}.time_ms: expected a number or null")
        if (e["time_ms"] is None) != (e["scored_by"] == "compile_time_model"):
            raise SchemaError(f"{w}.time_ms: null iff scored_by is compile_time_model")
        if not isinstance(e["validated"], bool):
            raise SchemaError(f"{w}.validated: expected a boolean")
        _check_keys(e["correctness"], ("cosine", "max_rel_err", "pcc"), w + ".correctness")
        for k in ("cosine", "max_rel_err", "pcc"):
            if not _is_num(e["correctness"][k]):
                raise SchemaError(f"{w}.correctness.{k}: expected a number")
    return doc


def load(path):
    with open(path) as f:
        return validate(json.load(f))


def save(doc, path):
    validate(doc)
    with open(path, "w") as f:
        json.dump(doc, f, indent=2)
        f.write("\n")


def entry(gpu, op, M, N, K, best, time_ms, validated, correctness, dtype="bf16"):
    return {"gpu": gpu, "op": op, "shape": {"M": M, "N": N, "K": K, "dtype": dtype},
            "best": {k: int(best[k]) for k in CONFIG_FIELDS},
            "scored_by": "measure" if time_ms is not None else "compile_time_model",
            "time_ms": time_ms, "validated": bool(validated),
            "correctness": {k: float(correctness[k]) for k in ("cosine", "max_rel_err", "pcc")}}


def merge(doc, new_entries):
    """Replace entries with the same (gpu, op, shape) key, append the rest."""
    key = lambda e: (e["gpu"], e["op"], e["shape"]["M"], e["shape"]["N"], e["shape"]["K"],  # noqa
                     e["shape"]["dtype"])
    keep = {key(e): e for e in doc.get("entries", [])}
    for e in new_entries:
        keep[key(e)] = e
    return {"version": 1, "entries": list(keep.values())}


# --------------------------------------------------------- runtime access --
def _cfg_array(c):
    return (ctypes.c_int * 7)(*[int(c[k]) for k in CONFIG_FIELDS])


def runtime_load(path):
    """Load a cache file into the C runtime; returns the entry count."""
    from ._lib import lib
    err = ctypes.create_string_buffer(512)
    n = lib().pkb200_tuning_load(path.encode(), err, 512)
    if n < 0:
        raise SchemaError(err.value.decode())
    return n


def runtime_select(op, M, N, K):
    """(source, config) the runtime would use: source 0 default, 1 cache, 2 forced."""
    from ._lib import lib
    out = (ctypes.c_int * 7)()
    src = lib().pkb200_gemm_select(op.encode(), M, N, K, out)
    if src < 0:
        raise ValueError(f"unknown op {op!r}")
    return src, dict(zip(CONFIG_FIELDS, list(out)))


def device_arch():
    from ._lib import lib
    buf = ctypes.create_string_buffer(32)
    lib().pkb200_device_arch(buf, 32)
    return buf.value.decode()


# --------------------------------------------------------------- autotune --
def _metrics(a, r):
    import torch
    a = a.double().flatten()
    r = r.double().flatten()
    cos = float(torch.dot(a, r) / (a.norm() * r.norm()).clamp_min(1e-300))
    rel = float(((a - r).abs() / (r.abs() + 1e-6)).max())
    ac, rc = a - a.mean(), r - r.mean()
    pcc = float((ac * rc).sum() / (ac.norm() * rc.norm()).clamp_min(1e-300))
    return {"cosine": cos, "max_rel_err": rel, "pcc": pcc}


def autotune(op, M, N, K, iters=10, warmup=3, seed=0, inject_broken=False, report=None):
    """Time every ConfigSpace config for `op` at (M, N, K) on the current GPU and
    return cache entries (one per op/shape: the fastest validated config).
    Ops: matmul, fused_matmul_bias_gelu, matmul_bias_residual.

    `inject_broken` adds a fast-but-wrong candidate (it only fills the output),
    the negative path of the reference's autotuner (tools/polykernel-bench/
    bench.py `--inject-broken`): the correctness gate must reject it although
    it is the fastest. `report`, when a list, receives one dict per candidate
    (label, time_ms, validated, metrics)."""
    import torch

    from . import ops
    from ._lib import lib
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(K, N, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = (0.02 * torch.randn(N, device="cuda", generator=g)).to(torch.bfloat16)
    resid = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    run = {"matmul": lambda: ops.matmul(a, b),
           "fused_matmul_bias_gelu": lambda: ops.fused_matmul_bias_gelu(a, b, bias),
           "matmul_bias_residual": lambda: ops.matmul_bias_residual(a, b, bias, resid)}[op]
    ref32 = a.float() @ b.float()
    if op == "fused_matmul_bias_gelu":
        ref32 = torch.nn.functional.gelu(ref32 + bias.float())
    elif op == "matmul_bias_residual":
        ref32 = ref32 + bias.float() + resid.float()
    broken_out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    candidates = [(f"block_m={c['block_m']},block_n={c['block_n']},"
                   f"stages={c['shared_memory_stages']}", c, run)
                  for c in ConfigSpace.enumerate()]
    if inject_broken:
        candidates.append(("broken", None, lambda: broken_out.fill_(0.5)))
    results = []
    try:
        lib().pkb200_set_gemm_config(_cfg_array(DEFAULT))
        base = run()
        for label, cfg, fn in candidates:
            if cfg is not None and lib().pkb200_set_gemm_config(_cfg_array(cfg)) != 0:
                continue
            out = fn()
            torch.cuda.synchronize()
            m = _metrics(out.float(), ref32)
            ok = bool(torch.equal(out, base)) and m["cosine"] >= 0.999 and m["pcc"] >= 0.99
            for _ in range(warmup):
                fn()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            t = s.elapsed_time(e) / iters
            results.append((t, ok, cfg, m))
            if report is not None:
                report.append({"label": label, "time_ms": t, "validated": ok, "metrics": m})
    finally:
        lib().pkb200_set_gemm_config(None)
    valid = [r for r in results if r[1] and r[2] is not None]
    if not valid:
        return []
    t, _, cfg, m = min(valid, key=lambda r: r[0])
    return [entry(device_arch(), op, M, N, K, cfg, t, True, m)]


# --------------------------------------------------------------------- CLI --
def main(argv=None):
    """python -m polykernel_b200.tuning <command> ...

    enumerate [--limit N]        the pruned tcgen05 config space, one JSON object per line
                                 (the reference driver's `enumerate --limit N`)
    validate FILE...             schema-check cache files; exit 1 on the first error
    show FILE                    one line per entry: gpu op MxNxK best validated time
    autotune --op OP --shape M N K [--shape ...] --out FILE [--inject-broken]
                                 tune on this GPU and merge the validated winners into FILE
    """
    import argparse
    import json
    import os
    import sys
    ap = argparse.ArgumentParser(prog="python -m polykernel_b200.tuning")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p_en = sub.add_parser("enumerate")
    p_en.add_argument("--limit", type=int, default=None)
    p_va = sub.add_parser("validate")
    p_va.add_argument("files", nargs="+")
    p_sh = sub.add_parser("show")
    p_sh.add_argument("file")
    p_at = sub.add_parser("autotune")
    p_at.add_argument("--op", required=True,
                      choices=["matmul", "fused_matmul_bias_gelu", "matmul_bias_residual"])
    p_at.add_argument("--shape", nargs=3, type=int, action="append", required=True,
                      metavar=("M", "N", "K"))
    p_at.add_argument("--out", required=True)
    p_at.add_argument("--iters", type=int, default=10)
    p_at.add_argument("--inject-broken", action="store_true",
                      help="add a fast-but-wrong candidate; the gate must reject it")
    a = ap.parse_args(argv)
    if a.cmd == "enumerate":
        for c in ConfigSpace.enumerate(a.limit):
            print(json.dumps(c))
        return 0
    if a.cmd == "validate":
        for f in a.files:
            try:
                n = len(load(f)["entries"])
            except (OSError, ValueError) as e:
                print(f"{f}: {e}", file=sys.stderr)
                return 1
            print(f"{f}: ok ({n} entries)")
        return 0
    if a.cmd == "show":
        try:
            doc = load(a.file)
        except (OSError, ValueError) as e:
            print(f"{a.file}: {e}", file=sys.stderr)
            return 1
        for e in doc["entries"]:
            s, b = e["shape"], e["best"]
            print(f"{e['gpu']} {e['op']} {s['M']}x{s['N']}x{s['K']} {s['dtype']} "
                  f"block_n={b['block_n']} stages={b['shared_memory_stages']} "
                  f"validated={e['validated']} time_ms={e['time_ms']}")
        return 0
    doc = load(a.out) if os.path.exists(a.out) else {"version": 1, "entries": []}
    for M, N, K in a.shape:
        report = []
        found = autotune(a.op, M, N, K, iters=a.iters, inject_broken=a.inject_broken,
                         report=report)
        for r in report:
            print(json.dumps({"op": a.op, "shape": [M, N, K], **{k: r[k] for k in
                              ("label", "time_ms", "validated")}}))
        if not found:
            print(f"{a.op} {M}x{N}x{K}: no candidate passed the correctness gate",
                  file=sys.stderr)
            return 1
        doc = merge(doc, found)
    save(doc, a.out)
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
