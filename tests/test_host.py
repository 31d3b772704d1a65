"""Host-side contract of the b200 package (runs without a GPU).

Configuration validation, parameter layout and initialisation identical to the
reference, cache dataclasses, and the C-ABI library: it loads and exports
every entry point that include/gpa_b200.h declares.  No compute call is made.
"""
from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

import oracle
from cases import CASES, build, params_digest
from check_oracle import load as load_golden
from gpa_b200 import DenseGPA, GPAConfig, GPAState, LevelState, RelationState
from gpa_b200 import _lib
from gpa_b200.state import tensors

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_config_accepts_default_flags_and_rejects_unimplemented_operators():
    GPAConfig(heads=16, key_dim=128, value_dim=128, slots=(64, 64, 64, 128), chunk_size=64)
    GPAConfig(positional_mode="none", chunk_size=1)
    GPAConfig(paper_product_read=True)
    GPAConfig(paper_product_read=True, relation_marginal=True)
    GPAConfig(positional_mode="moments")
    for bad in (dict(positional_mode="moments", key_dim=31), dict(rsa_update=True),
                dict(relation_marginal=True), dict(control_dim=4), dict(slot_feature="tanh"),
                dict(balanced_bridge=True), dict(quadratic_features=True),
                dict(learn_read_scale=True), dict(shared_query_center=True),
                dict(chunk_size=65), dict(slots=(256,)), dict(key_dim=130), dict(slots=(4,) * 9),
                dict(backend="torch"), dict(backend="fla", chunk_size=64)):
        with pytest.raises(ValueError):
            GPAConfig(**bad)
    # reference validation conditions (src/gpa/attention.py:46-73)
    for bad in (dict(heads=0), dict(slots=()), dict(slots=(0,)), dict(beta_init=.95),
                dict(relation_beta_init=1.), dict(decay_init=0.), dict(read_scale=0.),
                dict(execution="bogus"), dict(positional_mode="x")):
        with pytest.raises(ValueError):
            GPAConfig(**bad)


@pytest.mark.parametrize("name", ["config1", "chunk64_f32"])
def test_initialisation_and_state_dict_match_reference(name):
    """Same names, shapes and values as the reference model drawn from the same seed."""
    rec = load_golden(name)
    cfg, params, _ = build(name)
    torch.manual_seed(CASES[name]["seed"])
    model = DenseGPA(GPAConfig(**cfg))
    sd = model.state_dict()
    assert set(sd) == set(params)
    for key in params:
        assert sd[key].shape == params[key].shape, key
    if CASES[name].get("reference_init"):
        assert params_digest(sd) == rec["params_sha256"]
    model.load_state_dict(params, strict=True)


def test_cache_dataclasses_layout():
    cfg = GPAConfig(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=3)
    model = DenseGPA(cfg)
    st = model.initial_state(5)
    assert isinstance(st, GPAState) and isinstance(st.levels[0], LevelState)
    assert isinstance(st.relations[0], RelationState)
    assert [(r.source, r.target) for r in st.relations] == list(model.edges)
    assert st.levels[0].inner.shape == (5, 2, 4, 3) and st.levels[2].outer.shape == (5, 2, 4, 3)
    assert st.relations[1].memory.shape == (5, 2, 3, 4)
    ocfg = oracle.OracleConfig(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=3)
    ost = oracle.initial_state(ocfg, {k: v for k, v in model.state_dict().items()}, 5, torch.float32)
    assert [t.shape for t in tensors(st)] == [t.shape for t in oracle.tensors_of(ost)]
    assert st.numel() == sum(t.numel() for t in oracle.tensors_of(ost))
    assert not any(t.requires_grad for t in tensors(st.detach()))


def test_no_cpu_fallback():
    model = DenseGPA(GPAConfig(heads=2, key_dim=4, value_dim=3, slots=(3, 2), chunk_size=3))
    x = torch.randn(1, 4, 2, 4)
    with pytest.raises(ValueError, match="CUDA"):
        model(x, x, torch.randn(1, 4, 2, 3))


def _declared_functions():
    text = open(os.path.join(ROOT, "include", "gpa_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|long long)\s+(gpa_b200_\w+)\s*\(",
                                 text, re.M)))


def test_library_exports_every_declared_entry_point():
    if not os.path.exists(_lib.LIB_PATH):
        from gpa_b200.build import build as build_lib
        build_lib()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared_functions()
    assert set(declared) == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    loaded = _lib.load()
    assert loaded.gpa_b200_abi_version() == _lib.ABI_VERSION


def test_workspace_queries_and_argument_errors():
    lib = _lib.load()
    d = _lib.GpaDims()
    d.batch, d.length, d.heads, d.key_dim, d.value_dim, d.levels = 8, 512, 16, 128, 128, 4
    for j, m in enumerate((64, 64, 64, 128)):
        d.slots[j] = m
    d.chunk_size, d.chunk_offset, d.input_dtype = 64, 0, 1
    d.read_scale, d.query_scale, d.beta_max = 1., 1 / 16, .9
    assert lib.gpa_b200_saved_bytes(d) > 0 and lib.gpa_b200_scratch_bytes(d) > 0
    d.chunk_offset = 64
    assert lib.gpa_b200_saved_bytes(d) == 0
    d.chunk_offset = 0
    rc = lib.gpa_b200_forward(d, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 1
    buf = ctypes.create_string_buffer(256)
    assert lib.gpa_b200_last_error(buf, 256) == 1 and b"params" in buf.value
    with pytest.raises(ValueError, match="params"):
        _lib.check(rc, "gpa_b200_forward")
    d.reader_mode = 3  # beyond GPA_B200_READER_MARGINAL
    rc = lib.gpa_b200_forward(d, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 1 and lib.gpa_b200_last_error(buf, 256) == 1 and b"reader_mode" in buf.value


def test_bench_layer_workspaces_fit_one_b200():
    """The forward's saved buffer and the backward scratch of the benched training step (B=8,
    T=8192, H=16, 128/128, slots 64/64/64/128, chunk 64, bf16) leave most of a 180 GB B200 to the
    caller's tensors; a width above the supported 128 reports no size (unsupported)."""
    lib = _lib.load()
    d = _lib.GpaDims()
    d.batch, d.length, d.heads, d.key_dim, d.value_dim, d.levels = 8, 8192, 16, 128, 128, 4
    for j, m in enumerate((64, 64, 64, 128)):
        d.slots[j] = m
    d.chunk_size, d.chunk_offset, d.input_dtype = 64, 0, 1
    d.read_scale, d.query_scale, d.beta_max = 1., 1 / 16, .9
    saved, scratch = lib.gpa_b200_saved_bytes(d), lib.gpa_b200_scratch_bytes(d)
    io = 7 * 8 * 8192 * 16 * 128 * 2  # q, k, v, out and dq, dk, dv in bf16
    assert 0 < saved + scratch + io < 110e9
    d.slots[3] = 256
    assert lib.gpa_b200_saved_bytes(d) == 0 and lib.gpa_b200_scratch_bytes(d) == 0


def test_umma_selftest_rejects_unsupported_shapes_on_the_host():
    """Shape checks run before any CUDA call, so they answer without a GPU."""
    lib = _lib.load()
    for shape in ((129, 128, 64, 64), (64, 96, 64, 64), (64, 128, 8, 64), (64, 128, 64, 40),
                  (64, 128, 64, 256)):
        rc = lib.gpa_b200_umma_selftest(*shape, 0, 0, 0, 1, 1, 1, 1, 1, None)
        assert rc == 2, shape
    # the 16-lane read is for M = 64 with N a multiple of 16; unknown flags are refused
    for shape, flags in (((64, 128, 64, 64), 2), ((64, 64, 40, 64), 2), ((64, 64, 64, 64), 4)):
        rc = lib.gpa_b200_umma_selftest(*shape, 0, 0, flags, 1, 1, 1, 1, 1, None)
        assert rc == 2, (shape, flags)
