"""Host-side tests of libj1 (no GPU needed).

* The built library exports every function include/j1.h declares, and nothing else.
* ModelConfig parsing and its error messages follow src/config.rs:43-96; checkpoint
  checks follow src/weights.rs:51-89 (Git-LFS pointer, F32 only, shapes) and
  src/engine.rs:97-99 (INT8 markers); these run before any device work.
* Device strings follow Device::from_str (src/engine.rs:20-31); "cpu" is refused
  because libj1 has no CPU fallback.
* The micro-batch planner matches Engine::batches (src/engine.rs:191-210).
"""
import json
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import julia1 as j1
from julia1 import synthetic
from conftest import ROOT, has_gpu

HEADER = os.path.join(ROOT, "include", "j1.h")
TINY = dict(hidden=256, heads=4, layers=2, intermediate=256, vocab=300, max_positions=256, head_layers=1)


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"J1_API\s+[\w\s\*]+?\b(j1_\w+)\s*\(", text)))


def test_library_exports_exactly_the_header():
    declared = header_functions()
    assert len(declared) >= 25
    out = subprocess.run(["nm", "-D", "--defined-only", j1.LIB_PATH], capture_output=True, text=True, check=True)
    exported = sorted(l.split()[-1] for l in out.stdout.splitlines() if " T " in l)
    assert exported == declared
    assert sorted(j1.EXPORTS) == declared
    L = j1.lib()
    for name in declared:
        assert hasattr(L, name)


def test_version_and_status_names():
    L = j1.lib()
    assert L.j1_version().decode().startswith("libj1")
    for code, name in enumerate(j1.STATUS_NAMES):
        assert L.j1_status_name(code).decode() == name


@pytest.fixture(scope="module")
def tiny_ckpt(tmp_path_factory):
    return synthetic.write_checkpoint(str(tmp_path_factory.mktemp("tiny")), seed=1, **TINY)


def test_config_load(tiny_ckpt):
    c = j1.load_config(tiny_ckpt)
    assert (c.hidden, c.heads, c.head_dim, c.layers, c.intermediate) == (256, 4, 64, 2, 256)
    assert (c.half_window, c.vocab, c.max_positions, c.head_layers, c.head_heads, c.head_ff) == \
           (64, 300, 256, 1, 4, 1024)
    assert c.n_global == 1  # i % 3 == 0 for i in {0, 1}
    assert abs(c.norm_eps - 1e-5) < 1e-12


def _copy(src, dst, edit_enc=None, edit_julia=None):
    shutil.copytree(src, dst)
    if edit_enc:
        p = os.path.join(dst, "encoder", "config.json")
        d = json.load(open(p))
        edit_enc(d)
        json.dump(d, open(p, "w"))
    if edit_julia:
        p = os.path.join(dst, "julia_config.json")
        d = json.load(open(p))
        edit_julia(d)
        json.dump(d, open(p, "w"))
    return dst


@pytest.mark.parametrize("edit_enc,edit_julia,msg", [
    (None, lambda d: d.update(format_version=2), "Unsupported Julia checkpoint format"),
    (None, lambda d: d.update(weight_dtype="int8"), "Only float32 Julia checkpoints are supported"),
    (lambda d: d.update(model_type="bert"), None, "Encoder must be ModernBERT"),
    (lambda d: d.update(attention_bias=True), None, "Unsupported encoder setting attention_bias"),
    (lambda d: d.update(hidden_activation="silu"), None, "Unsupported encoder activation"),
    (lambda d: d.update(num_attention_heads=2), None, "Runtime kernels require head_dim 64"),
    (lambda d: d.update(layer_types=["full_attention"]), None, "layer_types must list every layer"),
    (lambda d: d.pop("vocab_size"), None, "config is missing vocab_size"),
    (None, lambda d: d.pop("head_layers"), "config is missing head_layers"),
])
def test_config_errors(tiny_ckpt, tmp_path, edit_enc, edit_julia, msg):
    root = _copy(tiny_ckpt, str(tmp_path / "c"), edit_enc, edit_julia)
    with pytest.raises(j1.J1Error) as e:
        j1.load_config(root)
    assert e.value.status == j1.IO and msg in str(e.value)


def test_rope_parameters_and_layer_types(tiny_ckpt, tmp_path):
    def edit(d):
        d["layer_types"] = ["sliding_attention", "full_attention"]
        d["rope_parameters"] = {"full_attention": {"rope_type": "default", "rope_theta": 5e5},
                                "sliding_attention": {"rope_type": "default", "rope_theta": 1e4}}
    root = _copy(tiny_ckpt, str(tmp_path / "c"), edit)
    c = j1.load_config(root)
    # `global` still follows i % every (src/config.rs:84-85); theta follows layer_types
    assert c.n_global == 1


def test_checkpoint_errors_before_any_device_work(tiny_ckpt, tmp_path):
    # Git-LFS pointer instead of weights
    root = _copy(tiny_ckpt, str(tmp_path / "lfs"))
    open(os.path.join(root, "model.safetensors"), "w").write("version https://git-lfs.github.com/spec/v1\noid x\n")
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(root, 0)
    assert e.value.status == j1.IO and "Git LFS" in str(e.value)
    # INT8 checkpoint marker
    root = _copy(tiny_ckpt, str(tmp_path / "int8"))
    open(os.path.join(root, "quantization.json"), "w").write("{}")
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(root, 0)
    assert e.value.status == j1.UNSUPPORTED and "INT8" in str(e.value)
    # a tensor with the wrong shape
    root = str(tmp_path / "shape")
    synthetic.write_checkpoint(root, seed=1, **dict(TINY, vocab=301))
    p = os.path.join(root, "encoder", "config.json")
    d = json.load(open(p))
    d["vocab_size"] = 300
    json.dump(d, open(p, "w"))
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(root, 0)
    assert e.value.status == j1.IO and "tok_embeddings.weight: expected shape" in str(e.value)
    # missing checkpoint
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(str(tmp_path / "nothing"), 0)
    assert e.value.status == j1.IO


def test_unsupported_shapes(tmp_path):
    root = synthetic.write_checkpoint(str(tmp_path / "h640"), seed=1, **dict(TINY, hidden=640, heads=10))
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(root, 0)
    assert e.value.status == j1.UNSUPPORTED and "head_dim 64" in str(e.value)
    root = synthetic.write_checkpoint(str(tmp_path / "nohead"), seed=1, **dict(TINY, head_layers=0))
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(root, 0)
    assert e.value.status == j1.UNSUPPORTED


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_model_create_without_gpu(tiny_ckpt):
    with pytest.raises(j1.J1Error) as e:
        j1.CudaModel(tiny_ckpt, 0)
    assert e.value.status == j1.CUDA and "CUDA device unavailable" in str(e.value)


def test_device_strings(tiny_ckpt):
    assert j1.Device.parse("cuda") == j1.Device("cuda", 0)
    assert j1.Device.parse("cuda:3") == j1.Device("cuda", 3)
    for bad in ("gpu", "cuda:", "cuda:x", "CUDA"):
        with pytest.raises(j1.J1Error):
            j1.Device.parse(bad)
    with pytest.raises(j1.J1Error) as e:
        j1.Engine.load(tiny_ckpt, j1.EngineOptions(device="cpu"))
    assert e.value.status == j1.UNSUPPORTED and "no CPU fallback" in str(e.value)


def reference_batches(lens, batch_size, max_tokens):
    """Engine::batches (src/engine.rs:191-210) restated."""
    order = sorted(range(len(lens)), key=lambda i: lens[i])  # Rust sort_by_key is stable
    out, group, tokens = [], [], 0
    for i in order:
        n = lens[i]
        if group and (len(group) == batch_size or tokens + n > max_tokens):
            out.append(group)
            group, tokens = [], 0
        group.append(i)
        tokens += n
    if group:
        out.append(group)
    return out


@pytest.mark.parametrize("seed", range(5))
@pytest.mark.parametrize("batch_size,max_tokens,devices", [(16, 65536, 1), (3, 1000, 2), (256, 131072, 8),
                                                           (1, 10, 3)])
def test_plan_matches_engine_batches(seed, batch_size, max_tokens, devices):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 1200, size=int(rng.integers(1, 300))).tolist()
    lens[::7] = [lens[0]] * len(lens[::7])  # ties keep input order
    batches, dev = j1.plan_batches(lens, batch_size, max_tokens, devices)
    assert batches == reference_batches(lens, batch_size, max_tokens)
    load = [0] * devices
    for b, d in zip(batches, dev):
        assert d == int(np.argmin(load))  # greedy: fewest tokens so far, lowest index on ties
        load[d] += sum(lens[i] for i in b)


def test_plan_errors():
    with pytest.raises(j1.J1Error):
        j1.plan_batches([1, 2], 0, 100, 1)
    assert j1.plan_batches([], 4, 100, 2) == ([], [])


def test_null_handles_are_rejected():
    L = j1.lib()
    assert L.j1_model_forward_many(None, 0, None, None) == j1.INVALID_ARG
    assert L.j1_model_launch(None) == j1.INVALID_ARG
    assert L.j1_engine_logits_encoded(None, 0, None, None, None, None, None, None) == j1.INVALID_ARG
    assert "NULL" in j1.last_error()


def test_python_constants_match_the_header():
    """The Python mirror's status codes, status names and fault kinds are the header's enums."""
    text = open(HEADER, encoding="utf-8").read()
    values = {name: int(v) for name, v in re.findall(r"\b(J1_(?:OK|ERR_[A-Z_]+|FAULT_[A-Z_]+))\s*=\s*(\d+)", text)}
    statuses = {k: v for k, v in values.items() if k == "J1_OK" or k.startswith("J1_ERR_")}
    assert statuses, "no status enum found"
    for name, v in statuses.items():
        assert getattr(j1, "OK" if name == "J1_OK" else name[len("J1_ERR_"):]) == v, name
        assert j1.STATUS_NAMES[v] == name
    assert len(j1.STATUS_NAMES) == len(statuses)
    faults = {k: v for k, v in values.items() if k.startswith("J1_FAULT_")}
    assert faults
    for name, v in faults.items():
        assert getattr(j1, name[len("J1_"):]) == v, name
