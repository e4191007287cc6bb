"""Loader, compatibility rules and call routing, without a GPU or a real library.

``relmo_b200.ops.mp_runtime`` (Policy, BuildInfo, check_compat, Library) and
``relmo_b200.ops.mp_dispatch.route`` are exercised with fake torch modules and
fake libraries: the environment settings relmo defines, the version / CUDA-tag
rules, one-time loading with the first failure remembered, and the routing
rule (CUDA always the library, no GPU fallback; CPU the library when usable,
else the Python formulas or an error).
"""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import pytest

from relmo_b200.ops import mp_dispatch, mp_runtime
from relmo_b200.ops.mp_constants import REQUIRED_NAMESPACE_OPS
from relmo_b200.ops.mp_runtime import BuildInfo, Library, Policy, check_compat

# ---- Policy ---------------------------------------------------------------------------------


def test_policy_defaults() -> None:
    assert Policy.from_env({}) == Policy(enabled=True, on_unavailable="python", version_policy="forward")


@pytest.mark.parametrize("word", ["0", "false", "No", " off "])
def test_policy_disable_words(word: str) -> None:
    assert Policy.from_env({"RELM_MP_ENABLE": word}).enabled is False


@pytest.mark.parametrize("word", ["1", "yes", "on", "anything"])
def test_policy_other_words_enable(word: str) -> None:
    assert Policy.from_env({"RELM_MP_ENABLE": word}).enabled is True


def test_policy_choices_and_unknown_values() -> None:
    p = Policy.from_env({"RELM_MP_FALLBACK": "ERROR", "RELM_MP_TORCH_VERSION_POLICY": "strict"})
    assert (p.on_unavailable, p.version_policy) == ("error", "strict")
    q = Policy.from_env({"RELM_MP_FALLBACK": "maybe", "RELM_MP_TORCH_VERSION_POLICY": "loose"})
    assert (q.on_unavailable, q.version_policy) == ("python", "forward")


def test_policy_reads_the_process_environment(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("RELM_MP_ENABLE", "off")
    assert Policy.from_env().enabled is False


# ---- BuildInfo / check_compat -------------------------------------------------------------


def test_build_info_parsing_keeps_extra_keys() -> None:
    info = BuildInfo.parse("build_torch=2.11.0;build_cuda_tag=cu128;abi_target=2.11;abi_lane=nonstable;arch=sm_100a;")
    assert info.torch_version == "2.11.0" and info.cuda_tag == "cu128"
    assert info.fields["arch"] == "sm_100a"
    assert mp_runtime.parse_build_info("a=1;junk;b = 2") == {"a": "1", "b": "2"}


def test_build_info_without_torch_version_is_rejected() -> None:
    with pytest.raises(RuntimeError, match="missing build_torch"):
        check_compat(BuildInfo.parse("build_cuda_tag=cpu"), "2.11.0", "cpu", "forward")


def _info(torch_v: str, tag: str = "cpu") -> BuildInfo:
    return BuildInfo.parse(f"build_torch={torch_v};build_cuda_tag={tag}")


def test_same_major_minor_is_silent(recwarn) -> None:
    check_compat(_info("2.11.0"), "2.11.3+cu128", "cu128", "strict")
    assert not [w for w in recwarn if issubclass(w.category, RuntimeWarning)]


def test_forward_policy_warns_on_newer_minor() -> None:
    with pytest.warns(RuntimeWarning, match="version drift"):
        check_compat(_info("2.10.1"), "2.11.0", "cpu", "forward")


def test_strict_policy_rejects_minor_drift() -> None:
    with pytest.raises(RuntimeError, match="Expected matching major.minor"):
        check_compat(_info("2.10.1"), "2.11.0", "cpu", "strict")


def test_older_runtime_and_other_major_are_rejected() -> None:
    with pytest.raises(RuntimeError, match="older than the build torch"):
        check_compat(_info("2.11.0"), "2.10.0", "cpu", "forward")
    with pytest.raises(RuntimeError, match="major version mismatch"):
        check_compat(_info("2.11.0"), "3.0.0", "cpu", "forward")


def test_cuda_tag_rules() -> None:
    with pytest.raises(RuntimeError, match="CUDA tag mismatch"):
        check_compat(_info("2.11.0", "cu128"), "2.11.0", "cu126", "forward")
    check_compat(_info("2.11.0", "cpu"), "2.11.0", "cu128", "forward")  # a CPU build runs anywhere
    assert mp_runtime.cuda_tag_of("12.8") == "cu128" and mp_runtime.cuda_tag_of(None) == "cpu"


# ---- Library -----------------------------------------------------------------------------


def _namespace(build_info: str = "build_torch=2.11.0;build_cuda_tag=cpu", ops=REQUIRED_NAMESPACE_OPS):
    ns = SimpleNamespace(**{op: (lambda *a: None) for op in ops})
    ns.build_info = lambda: build_info
    return ns


class FakeTorch:
    def __init__(self, namespaces: dict[str, SimpleNamespace], version: str = "2.11.0", cuda: str | None = None):
        self.__version__ = version
        self.version = SimpleNamespace(cuda=cuda)
        self.loads: list[str] = []
        outer = self

        class Ops:
            def load_library(self, path: str) -> None:
                outer.loads.append(Path(path).name)
                if Path(path).name not in namespaces:
                    raise OSError("cannot open shared object")
                self.relm_mp = namespaces[Path(path).name]

        self.ops = Ops()


def test_library_missing_is_reported_once() -> None:
    t = FakeTorch({})
    lib = Library(torch_module=t, candidates=lambda: [])
    with pytest.raises(RuntimeError, match="Could not find relm_mp custom op library"):
        lib.load()
    with pytest.raises(RuntimeError):
        lib.load()
    assert lib.usable() is False and t.loads == []


def test_library_skips_incomplete_candidates() -> None:
    partial = _namespace(ops=("fanout_scatter",))
    t = FakeTorch({"a.so": partial, "b.so": _namespace()})
    lib = Library(torch_module=t, candidates=lambda: [Path("/x/a.so"), Path("/x/b.so")])
    lib.load()
    assert lib.path == Path("/x/b.so") and t.loads == ["a.so", "b.so"]
    lib.load()  # no second attempt
    assert t.loads == ["a.so", "b.so"]
    assert hasattr(lib.ops(), "fanin_reduce")


def test_library_incomplete_everywhere_names_the_missing_ops() -> None:
    t = FakeTorch({"a.so": _namespace(ops=("fanout_scatter",))})
    lib = Library(torch_module=t, candidates=lambda: [Path("a.so")])
    with pytest.raises(RuntimeError, match="lacks .*fanin_reduce"):
        lib.load()


def test_library_compat_failure_makes_it_unusable(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.delenv("RELM_MP_TORCH_VERSION_POLICY", raising=False)
    t = FakeTorch({"a.so": _namespace("build_torch=2.11.0;build_cuda_tag=cu128")}, cuda="12.6")
    lib = Library(torch_module=t, candidates=lambda: [Path("a.so")])
    assert lib.usable() is False
    assert "CUDA tag mismatch" in str(lib.error)


def test_package_library_candidates() -> None:
    names = [p.name for p in mp_runtime.candidate_libraries()]
    assert "relm_mp_ops.so" in names
    assert "librelm_mp_b200.so" not in names  # the C-ABI library is not a torch op library


# ---- routing ---------------------------------------------------------------------------------


class FakeLibrary:
    def __init__(self, ok: bool, ops=("fanout_scatter", "fanin_reduce")):
        self.ok = ok
        self.ns = SimpleNamespace(**{op: (lambda *a: "custom") for op in ops})

    def load(self):
        if not self.ok:
            raise RuntimeError("relm_mp library unavailable: no .so")
        return self

    def ops(self):
        self.load()
        return self.ns

    def has_op(self, op_name: str) -> bool:
        return hasattr(self.ops(), op_name)


CUDA_T = SimpleNamespace(is_cuda=True)
CPU_T = SimpleNamespace(is_cuda=False)


@pytest.fixture
def env(monkeypatch: pytest.MonkeyPatch):
    for name in ("RELM_MP_ENABLE", "RELM_MP_FALLBACK"):
        monkeypatch.delenv(name, raising=False)

    def use(lib: FakeLibrary, **envvars: str) -> None:
        monkeypatch.setattr(mp_dispatch, "library", lambda: lib)
        for k, v in envvars.items():
            monkeypatch.setenv(k, v)

    return use


def test_cuda_calls_go_to_the_library(env) -> None:
    env(FakeLibrary(True))
    assert mp_dispatch.route("fanin_reduce", CUDA_T) == mp_dispatch.CUSTOM


@pytest.mark.parametrize(
    "lib_ok,settings", [(True, dict(RELM_MP_ENABLE="0")), (False, dict()), (False, dict(RELM_MP_FALLBACK="python"))]
)
def test_cuda_calls_never_fall_back(env, lib_ok, settings) -> None:
    env(FakeLibrary(lib_ok), **settings)
    with pytest.raises(RuntimeError, match="no GPU fallback"):
        mp_dispatch.route("fanin_reduce", CUDA_T)


def test_cuda_call_of_an_op_the_library_lacks_raises(env) -> None:
    env(FakeLibrary(True, ops=("fanin_reduce",)))
    with pytest.raises(RuntimeError, match="not in the loaded relm_mp library"):
        mp_dispatch.route("fanout_scatter", CUDA_T)


def test_cpu_calls_use_the_library_when_usable(env) -> None:
    env(FakeLibrary(True))
    assert mp_dispatch.route("fanout_scatter", CPU_T) == mp_dispatch.CUSTOM
    assert mp_dispatch.call("fanout_scatter", 1, 2, tensor=CPU_T, python=lambda *a: "python") == "custom"


def test_cpu_calls_fall_back_when_disabled_or_unusable(env) -> None:
    env(FakeLibrary(True), RELM_MP_ENABLE="false")
    assert mp_dispatch.route("fanin_reduce", CPU_T) == mp_dispatch.PYTHON
    env(FakeLibrary(False), RELM_MP_ENABLE="1")
    assert mp_dispatch.route("fanin_reduce", CPU_T) == mp_dispatch.PYTHON
    assert mp_dispatch.call("fanin_reduce", 1, tensor=CPU_T, python=lambda *a: "python") == "python"


def test_cpu_calls_of_missing_ops_fall_back(env) -> None:
    env(FakeLibrary(True, ops=("fanin_reduce",)))
    assert mp_dispatch.route("fanout_pack_multi", CPU_T) == mp_dispatch.PYTHON


def test_error_policy_raises_instead_of_falling_back(env) -> None:
    env(FakeLibrary(False), RELM_MP_FALLBACK="error")
    with pytest.raises(RuntimeError, match="Custom mp op fanin_reduce is unavailable"):
        mp_dispatch.route("fanin_reduce", CPU_T)
    # a disabled library is a choice, not a failure: the formulas run
    env(FakeLibrary(False), RELM_MP_FALLBACK="error", RELM_MP_ENABLE="0")
    assert mp_dispatch.route("fanin_reduce", CPU_T) == mp_dispatch.PYTHON
