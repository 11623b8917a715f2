"""Tuning cache + runtime selection (lib/Autotune + lib/Runtime/KernelCache
semantics): schema rules shared by the Python writer and the C loader, config
space pruning, selection of validated entries only. CPU except the autotune test."""
import copy
import ctypes
import json

import pytest

from polykernel_b200 import tuning as T
from polykernel_b200._lib import lib

GOOD = {"version": 1, "entries": [T.entry("sm_100", "matmul", 256, 512, 1024,
                                          dict(T.DEFAULT, block_n=128, shared_memory_stages=6),
                                          0.0123, True,
                                          {"cosine": 1.0, "max_rel_err": 0.0, "pcc": 1.0})]}


def _c_load(tmp_path, doc_text):
    p = tmp_path / "cache.json"
    p.write_text(doc_text)
    err = ctypes.create_string_buffer(512)
    n = lib().pkb200_tuning_load(str(p).encode(), err, 512)
    return n, err.value.decode()


def test_roundtrip_python_and_c(tmp_path):
    T.save(GOOD, tmp_path / "c.json")
    assert T.load(tmp_path / "c.json") == GOOD
    n, err = _c_load(tmp_path, json.dumps(GOOD))
    assert n == 1 and err == ""
    lib().pkb200_tuning_clear()


@pytest.mark.parametrize("mutate,fragment", [
    (lambda d: d.update(version=2), "version"),
    (lambda d: d.update(extra=1), "unknown field"),
    (lambda d: d["entries"][0].pop("validated"), "missing field"),
    (lambda d: d["entries"][0]["best"].update(block_n="128"), "block_n"),
    (lambda d: d["entries"][0].update(time_ms=None), "time_ms"),
    (lambda d: d["entries"][0].update(scored_by="guess"), "scored_by"),
    (lambda d: d["entries"][0]["shape"].update(M=1.5), "shape.M"),
    (lambda d: d["entries"][0]["correctness"].update(pcc=True), "pcc"),
])
def test_schema_errors_rejected_by_both(tmp_path, mutate, fragment):
    bad = copy.deepcopy(GOOD)
    mutate(bad)
    with pytest.raises(T.SchemaError, match=fragment.split(".")[-1]):
        T.validate(bad)
    n, err = _c_load(tmp_path, json.dumps(bad))
    assert n == -1 and fragment.split(".")[-1] in err


def test_c_loader_rejects_malformed_json(tmp_path):
    n, err = _c_load(tmp_path, '{"version": 1, "entries": [')
    assert n == -1 and err
    n, err = _c_load(tmp_path, '{"version": 1, "entries": []} trailing')
    assert n == -1


def test_config_space_pruning():
    cfgs = T.ConfigSpace.enumerate()
    triples = {(c["block_m"], c["block_n"], c["shared_memory_stages"]) for c in cfgs}
    assert triples == T.COMPILED
    assert T.ConfigSpace.prune_reason(dict(T.DEFAULT, shared_memory_stages=5)) in (
        "shared memory", "no compiled variant")
    assert T.ConfigSpace.prune_reason(dict(T.DEFAULT, shared_memory_stages=8)) == "shared memory"
    assert T.ConfigSpace.prune_reason(dict(T.DEFAULT, unroll=4)) == "tmem columns"
    assert all(T.ConfigSpace.smem_bytes(c) <= T.SMEM_LIMIT for c in cfgs)


def test_selection_serves_validated_entries_for_this_arch_only(tmp_path):
    # Without a GPU the runtime detects arch "unknown"; entries keyed to it
    # exercise the matching rules (validated, gpu, op, exact shape).
    arch = T.device_arch()
    hit = T.entry(arch, "matmul", 256, 512, 1024, dict(T.DEFAULT, block_n=128), 0.01, True,
                  {"cosine": 1, "max_rel_err": 0, "pcc": 1})
    unvalidated = T.entry(arch, "fused_matmul_bias_gelu", 256, 512, 1024,
                          dict(T.DEFAULT, block_n=128), 0.01, False,
                          {"cosine": 0.5, "max_rel_err": 1, "pcc": 0.5})
    other_gpu = T.entry("sm_90", "matmul_bias_residual", 256, 512, 1024,
                        dict(T.DEFAULT, block_n=128), 0.01, True,
                        {"cosine": 1, "max_rel_err": 0, "pcc": 1})
    no_variant = T.entry(arch, "matmul_f32out", 256, 512, 1024,
                         dict(T.DEFAULT, block_n=64), 0.01, True,
                         {"cosine": 1, "max_rel_err": 0, "pcc": 1})
    path = tmp_path / "c.json"
    T.save({"version": 1, "entries": [hit, unvalidated, other_gpu, no_variant]}, path)
    assert T.runtime_load(str(path)) == 4
    try:
        src, cfg = T.runtime_select("matmul", 256, 512, 1024)
        assert src == 1 and cfg["block_n"] == 128
        assert T.runtime_select("fused_rmsnorm_matmul", 256, 512, 1024)[0] == 1  # alias
        assert T.runtime_select("matmul", 256, 512, 1023)[0] == 0                 # exact shape
        assert T.runtime_select("fused_matmul_bias_gelu", 256, 512, 1024)[0] == 0  # not validated
        assert T.runtime_select("matmul_bias_residual", 256, 512, 1024)[0] == 0    # other gpu
        assert T.runtime_select("matmul_f32out", 256, 512, 1024)[0] == 0           # no variant
        with pytest.raises(ValueError):
            T.runtime_select("softmax", 1, 1, 1)
    finally:
        lib().pkb200_tuning_clear()
    assert T.runtime_select("matmul", 256, 512, 1024)[0] == 0


def test_forced_config_validation():
    bad = (ctypes.c_int * 7)(128, 64, 64, 10, 8, 2, 4)
    assert lib().pkb200_set_gemm_config(bad) != 0
    good = T._cfg_array(dict(T.DEFAULT, block_n=128, shared_memory_stages=4))
    assert lib().pkb200_set_gemm_config(good) == 0
    try:
        src, cfg = T.runtime_select("matmul", 8, 8, 8)
        assert src == 2 and cfg["block_n"] == 128
    finally:
        lib().pkb200_set_gemm_config(None)
    assert T.runtime_select("matmul", 8, 8, 8)[0] == 0


@pytest.mark.gpu
def test_autotune_cache_roundtrip_on_gpu(cuda, tmp_path):
    import torch
    import polykernel_b200 as pk
    M, N, K = 512, 1024, 768
    entries = T.autotune("matmul", M, N, K, iters=3, warmup=1)
    assert len(entries) == 1 and entries[0]["validated"] and entries[0]["gpu"] == "sm_100"
    doc = T.merge({"version": 1, "entries": []}, entries)
    T.save(doc, tmp_path / "tuned.json")
    # force a non-default winner into the cache to prove the runtime serves it
    doc["entries"][0]["best"] = dict(T.DEFAULT, block_n=128, shared_memory_stages=6)
    T.save(doc, tmp_path / "tuned.json")
    assert T.runtime_load(str(tmp_path / "tuned.json")) == 1
    try:
        a = torch.randn(M, K, device="cuda").bfloat16()
        b = torch.randn(K, N, device="cuda").bfloat16()
        out = pk.ops.matmul(a, b)
        last = (ctypes.c_int * 7)()
        lib().pkb200_last_gemm_config(last)
        assert list(last)[1] == 128 and list(last)[6] == 6
    finally:
        lib().pkb200_tuning_clear()
    ref = pk.ops.matmul(a, b)          # default variant
    assert torch.equal(out, ref)       # same K order in every variant: bit-identical


@pytest.mark.gpu
@pytest.mark.parametrize("bm,bn,stages", sorted(T.COMPILED))
def test_every_compiled_variant_matches_default(cuda, bm, bn, stages):
    import torch
    import polykernel_b200 as pk
    g = torch.Generator(device="cuda").manual_seed(5)
    for (M, N, K) in ((300, 520, 256), (1024, 2048, 4096)):
        a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        b = (torch.randn(K, N, device="cuda", generator=g) / K ** 0.5).bfloat16()
        bias = torch.randn(N, device="cuda", generator=g).bfloat16()
        ref = pk.ops.fused_matmul_bias_gelu(a, b, bias)
        assert lib().pkb200_set_gemm_config(
            T._cfg_array(dict(T.DEFAULT, block_m=bm, block_n=bn,
                              shared_memory_stages=stages))) == 0
        try:
            out = pk.ops.fused_matmul_bias_gelu(a, b, bias)
        finally:
            lib().pkb200_set_gemm_config(None)
        assert torch.equal(out, ref), (bm, bn, stages, M, N, K)
    assert pk.device_error() == 0


@pytest.mark.gpu
def test_autotune_rejects_injected_broken_variant(cuda):
    """Negative path (the reference autotuner's --inject-broken): a candidate
    that only fills its output is the fastest, yet the correctness gate rejects
    it and the cache entry names a real tcgen05 config."""
    report = []
    entries = T.autotune("matmul", 2048, 2048, 2048, iters=5, warmup=2, inject_broken=True,
                         report=report)
    broken = [r for r in report if r["label"] == "broken"]
    assert broken and not broken[0]["validated"]
    assert broken[0]["time_ms"] <= min(r["time_ms"] for r in report)
    assert len(entries) == 1 and entries[0]["validated"]
    best = entries[0]["best"]
    assert (best["block_m"], best["block_n"], best["shared_memory_stages"]) in T.COMPILED


def test_cli_enumerate_validate_show(tmp_path, capsys):
    import json as _json
    assert T.main(["enumerate", "--limit", "2"]) == 0
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]
    assert len(lines) == 2
    assert all((_json.loads(ln)["block_m"], _json.loads(ln)["block_n"],
                _json.loads(ln)["shared_memory_stages"]) in T.COMPILED
               for ln in lines)
    doc = T.merge({"version": 1, "entries": []},
                  [T.entry("sm_100", "matmul", 256, 512, 1024, T.DEFAULT, 0.01, True,
                           {"cosine": 1.0, "max_rel_err": 0.0, "pcc": 1.0})])
    good = tmp_path / "good.json"
    T.save(doc, good)
    assert T.main(["validate", str(good)]) == 0
    assert "ok (1 entries)" in capsys.readouterr().out
    assert T.main(["show", str(good)]) == 0
    out = capsys.readouterr().out
    assert "sm_100 matmul 256x512x1024 bf16 block_n=256 stages=4 validated=True" in out
    bad = tmp_path / "bad.json"
    d = _json.loads(good.read_text())
    d["entries"][0]["validated"] = "yes"
    bad.write_text(_json.dumps(d))
    assert T.main(["validate", str(good), str(bad)]) == 1
    assert "validated" in capsys.readouterr().err
