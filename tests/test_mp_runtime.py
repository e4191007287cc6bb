"""Loader / compat / dispatch policy, with a fake torch (no GPU, no library).

The cases follow relmo's ``tests/python/test_mp_runtime.py`` (version drift
warn/reject 40-88, CUDA-tag mismatch 91-104, missing or incomplete library
121-151, dispatch env policy 154-185) on ``relmo_b200.ops.mp_runtime`` and
``mp_dispatch``, plus the B200 policy that CUDA tensors have no fallback.
"""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import pytest

from relmo_b200.ops import mp_dispatch, mp_runtime


@pytest.fixture(autouse=True)
def _reset_mp_runtime_state(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(mp_runtime, "_LIB_LOADED", False)
    monkeypatch.setattr(mp_runtime, "_LIB_LOAD_ERROR", None)
    monkeypatch.setattr(mp_runtime, "_BUILD_INFO_CACHE", None)
    monkeypatch.setattr(mp_runtime, "_RUNTIME_COMPAT_VALIDATED", False)


def _fake_torch(*, version: str, cuda: str | None = None, namespace: object | None = None):
    ops = SimpleNamespace(load_library=lambda path: None)
    if namespace is not None:
        ops.relm_mp = namespace
    return SimpleNamespace(__version__=version, version=SimpleNamespace(cuda=cuda), ops=ops)


def _patch(monkeypatch, namespace, version, cuda, policy=None):
    monkeypatch.setattr(mp_runtime, "torch", _fake_torch(version=version, cuda=cuda, namespace=namespace))
    monkeypatch.setattr(mp_runtime, "ensure_loaded", lambda: None)
    monkeypatch.setattr(mp_runtime, "ops_namespace", lambda: namespace)
    if policy is not None:
        monkeypatch.setattr(mp_runtime, "torch_version_policy", lambda: policy)


def test_runtime_env_parsing(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("RELM_MP_ENABLE", "false")
    monkeypatch.setenv("RELM_MP_FALLBACK", "error")
    monkeypatch.setenv("RELM_MP_TORCH_VERSION_POLICY", "strict")
    assert mp_runtime.env_bool_any(("RELM_MP_ENABLE",), True) is False
    assert mp_runtime.fallback_mode() == "error"
    assert mp_runtime.torch_version_policy() == "strict"


def test_forward_policy_warns_on_newer_minor(monkeypatch: pytest.MonkeyPatch) -> None:
    ns = SimpleNamespace(build_info=lambda: "build_torch=2.5.1;build_cuda_tag=cpu")
    _patch(monkeypatch, ns, "2.6.0", None, "forward")
    with pytest.warns(RuntimeWarning, match="version drift"):
        info = mp_runtime.assert_runtime_compat()
    assert info["build_torch"] == "2.5.1"


def test_strict_policy_rejects_minor_drift(monkeypatch: pytest.MonkeyPatch) -> None:
    ns = SimpleNamespace(build_info=lambda: "build_torch=2.5.1;build_cuda_tag=cpu")
    _patch(monkeypatch, ns, "2.6.0", None, "strict")
    with pytest.raises(RuntimeError, match="Expected matching major.minor"):
        mp_runtime.assert_runtime_compat()


def test_rejects_older_runtime(monkeypatch: pytest.MonkeyPatch) -> None:
    ns = SimpleNamespace(build_info=lambda: "build_torch=2.6.0;build_cuda_tag=cpu")
    _patch(monkeypatch, ns, "2.5.1", None, "forward")
    with pytest.raises(RuntimeError, match="runtime is older than the build torch"):
        mp_runtime.assert_runtime_compat()


def test_rejects_cuda_tag_mismatch(monkeypatch: pytest.MonkeyPatch) -> None:
    ns = SimpleNamespace(build_info=lambda: "build_torch=2.5.1;build_cuda_tag=cu124")
    _patch(monkeypatch, ns, "2.5.1", "12.1")
    with pytest.raises(RuntimeError, match="CUDA tag mismatch"):
        mp_runtime.assert_runtime_compat()


def test_extra_build_info_keys_are_ignored(monkeypatch: pytest.MonkeyPatch) -> None:
    ns = SimpleNamespace(
        build_info=lambda: "build_torch=2.11.0;build_cuda_tag=cu128;abi_target=2.11;abi_lane=nonstable;"
        "lib=relm_mp_b200;arch=sm_100a;kernel_cuda=12.9;abi=1"
    )
    _patch(monkeypatch, ns, "2.11.0+cu128", "12.8")
    assert mp_runtime.assert_runtime_compat()["arch"] == "sm_100a"


def test_available_false_when_compat_check_fails(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(mp_runtime, "torch", object())
    monkeypatch.setattr(mp_runtime, "ensure_loaded", lambda: None)
    monkeypatch.setattr(
        mp_runtime, "assert_runtime_compat", lambda: (_ for _ in ()).throw(RuntimeError("boom"))
    )
    assert mp_runtime.available() is False


def test_ensure_loaded_raises_when_library_is_missing(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(mp_runtime, "candidate_libraries", lambda: [])
    monkeypatch.setattr(mp_runtime, "torch", _fake_torch(version="2.5.1"))
    with pytest.raises(FileNotFoundError, match="Could not find relm_mp custom op library"):
        mp_runtime.ensure_loaded()


def test_ensure_loaded_raises_when_namespace_is_incomplete(monkeypatch: pytest.MonkeyPatch) -> None:
    class FakeOps:
        def __init__(self) -> None:
            self.relm_mp = SimpleNamespace(fanout_scatter=lambda *args: None)

        def load_library(self, path: str) -> None:
            del path

    monkeypatch.setattr(mp_runtime, "candidate_libraries", lambda: [Path("/tmp/fake.so")])
    monkeypatch.setattr(
        mp_runtime, "torch", SimpleNamespace(__version__="2.5.1", version=SimpleNamespace(cuda=None), ops=FakeOps())
    )
    with pytest.raises(RuntimeError, match="Failed to load relm_mp custom op library"):
        mp_runtime.ensure_loaded()


def test_candidate_libraries_glob_the_package_dir() -> None:
    names = [p.name for p in mp_runtime.candidate_libraries()]
    assert "relm_mp_ops.so" in names
    assert "librelm_mp_b200.so" not in names  # the C-ABI library is not a torch op library


def test_dispatch_disable_env_short_circuits(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("RELM_MP_ENABLE", "0")
    assert mp_dispatch.should_use_custom("fanout_scatter") is False


def test_dispatch_error_mode_raises_when_custom_unavailable(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.delenv("RELM_MP_ENABLE", raising=False)
    monkeypatch.setenv("RELM_MP_FALLBACK", "error")
    monkeypatch.setattr(
        mp_dispatch, "ensure_runtime_compat_once", lambda: (_ for _ in ()).throw(RuntimeError("missing custom op"))
    )
    with pytest.raises(RuntimeError, match="Custom mp op fanout_scatter is unavailable"):
        mp_dispatch.should_use_custom("fanout_scatter")


def test_gpu_path_has_no_fallback(monkeypatch: pytest.MonkeyPatch) -> None:
    """relmo fell back to Python on the GPU when the library was missing; relmo_b200 raises."""

    monkeypatch.delenv("RELM_MP_ENABLE", raising=False)
    monkeypatch.setenv("RELM_MP_FALLBACK", "python")
    monkeypatch.setattr(
        mp_dispatch, "ensure_runtime_compat_once", lambda: (_ for _ in ()).throw(RuntimeError("no library"))
    )
    with pytest.raises(RuntimeError, match="no GPU fallback"):
        mp_dispatch.require_gpu_custom("fanin_reduce")
    monkeypatch.setenv("RELM_MP_ENABLE", "0")
    with pytest.raises(RuntimeError, match="no GPU fallback"):
        mp_dispatch.require_gpu_custom("fanin_reduce")


def test_namespace_has_op_uses_loaded_namespace(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setattr(mp_dispatch, "torch", object())
    monkeypatch.setattr(mp_dispatch, "ensure_loaded", lambda: None)
    monkeypatch.setattr(mp_dispatch, "ops_namespace", lambda: SimpleNamespace(example_op=lambda *a: None))
    assert mp_dispatch.namespace_has_op("example_op") is True
    assert mp_dispatch.namespace_has_op("missing_op") is False
