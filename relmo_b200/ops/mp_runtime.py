"""Finding, loading and vetting the ``relm_mp`` torch library of this package.

Three pieces, each usable on its own:

* :class:`Policy` - the operator's settings, read from the environment. The
  variable names and their meanings are relmo's (``src/relmo/ops/mp_runtime.py``
  44-69), so a deployment configures this package the way it configured relmo:
  ``RELM_MP_ENABLE`` (default on), ``RELM_MP_FALLBACK=python|error`` (what a CPU
  call does when the library is unusable) and
  ``RELM_MP_TORCH_VERSION_POLICY=forward|strict``.
* :class:`BuildInfo` and :func:`check_compat` - the ``build_info()`` string of the
  library (``key=value;...``, mp_ops.cpp:3745-3749) and relmo's compatibility
  rules for it (mp_runtime.py:175-228): the torch major version must match; under
  ``strict`` the minor too; under ``forward`` a newer runtime minor is accepted
  with a warning and an older one rejected; a CUDA build must match the
  runtime's CUDA tag.
* :class:`Library` - one process-wide load of the first ``relm_mp_ops*.so`` /
  ``librelm_mp_ops*.so`` in the package directory (where relmo's loader looks,
  mp_runtime.py:97-125), accepted only when it registers every op of
  ``REQUIRED_NAMESPACE_OPS`` and passes the compat check. The outcome (loaded, or
  the error) is remembered, so a broken install costs one attempt.

relmo's CUDA variant switches (``RELM_MP_FANOUT_BWD_KERNEL``,
``RELM_MP_FANIN_LSE_FWD``) have no counterpart: each op has one tuned path.
"""

from __future__ import annotations

import os
import re
import sys
import threading
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Mapping

from .mp_constants import REQUIRED_NAMESPACE_OPS

try:
    import torch
except Exception as exc:  # pragma: no cover - environments without torch
    torch = None
    TORCH_IMPORT_ERROR: Exception | None = exc
else:
    TORCH_IMPORT_ERROR = None

NAMESPACE = "relm_mp"
OWN_NAMESPACE = "relm_mp_b200"  # ops of this package outside the reference schemas
LIBRARY_GLOBS = ("relm_mp_ops*.so", "librelm_mp_ops*.so")


def require_torch(feature_name: str) -> None:
    if torch is None:
        raise ModuleNotFoundError(f"{feature_name} requires torch.") from TORCH_IMPORT_ERROR


# ---- operator settings ---------------------------------------------------------------

_OFF_WORDS = frozenset({"0", "false", "no", "off"})


@dataclass(frozen=True)
class Policy:
    enabled: bool = True
    on_unavailable: str = "python"  # "python" | "error": CPU calls when the library is unusable
    version_policy: str = "forward"  # "forward" | "strict"

    @classmethod
    def from_env(cls, env: Mapping[str, str] | None = None) -> "Policy":
        env = os.environ if env is None else env

        def pick(name: str, allowed: tuple[str, ...], default: str) -> str:
            value = env.get(name, default).strip().lower()
            return value if value in allowed else default

        enabled_raw = env.get("RELM_MP_ENABLE")
        return cls(
            enabled=True if enabled_raw is None else enabled_raw.strip().lower() not in _OFF_WORDS,
            on_unavailable=pick("RELM_MP_FALLBACK", ("python", "error"), "python"),
            version_policy=pick("RELM_MP_TORCH_VERSION_POLICY", ("forward", "strict"), "forward"),
        )


# ---- build metadata and compatibility ---------------------------------------------------

_MAJOR_MINOR = re.compile(r"^(\d+)\.(\d+)")


def _major_minor(version: str) -> tuple[int, int]:
    m = _MAJOR_MINOR.match(version)
    if m is None:
        raise RuntimeError(f"Could not parse torch version {version!r}.")
    return int(m.group(1)), int(m.group(2))


@dataclass(frozen=True)
class BuildInfo:
    fields: dict[str, str] = field(default_factory=dict)

    @classmethod
    def parse(cls, text: str) -> "BuildInfo":
        pairs = (item.split("=", 1) for item in text.split(";") if "=" in item)
        return cls({k.strip(): v.strip() for k, v in pairs})

    @property
    def torch_version(self) -> str:
        value = self.fields.get("build_torch", "")
        if not value:
            raise RuntimeError("mp build metadata is missing build_torch.")
        return value

    @property
    def cuda_tag(self) -> str:
        return self.fields.get("build_cuda_tag", "cpu")


def parse_build_info(text: str) -> dict[str, str]:
    return dict(BuildInfo.parse(text).fields)


def cuda_tag_of(cuda_version: str | None) -> str:
    return f"cu{str(cuda_version).replace('.', '')}" if cuda_version else "cpu"


def check_compat(build: BuildInfo, runtime_torch: str, runtime_cuda_tag: str, version_policy: str) -> None:
    """Raise RuntimeError when the library cannot run under this torch; warn
    (RuntimeWarning) when it runs on a newer torch minor than it was built for."""

    built = build.torch_version
    b, r = _major_minor(built), _major_minor(runtime_torch)
    if b != r:
        if version_policy == "strict":
            raise RuntimeError(
                f"mp torch version mismatch: built against {built}, runtime is {runtime_torch}. "
                "Expected matching major.minor."
            )
        if b[0] != r[0]:
            raise RuntimeError(f"mp torch major version mismatch: built against {built}, runtime is {runtime_torch}.")
        if r < b:
            raise RuntimeError(
                f"mp torch runtime is older than the build torch: built against {built}, runtime is "
                f"{runtime_torch}. Rebuild against the older torch or upgrade the runtime torch."
            )
        warnings.warn(
            f"mp torch version drift: built against {built}, runtime is {runtime_torch}; accepted under "
            "RELM_MP_TORCH_VERSION_POLICY=forward (tested compatibility, not a guaranteed ABI).",
            RuntimeWarning,
            stacklevel=3,
        )
    if build.cuda_tag != "cpu" and build.cuda_tag != runtime_cuda_tag:
        raise RuntimeError(f"mp CUDA tag mismatch: built for {build.cuda_tag}, runtime is {runtime_cuda_tag}.")


# ---- the library ----------------------------------------------------------------------------


def package_dir() -> Path:
    return Path(__file__).resolve().parent.parent


def candidate_libraries(directory: Path | None = None) -> list[Path]:
    directory = package_dir() if directory is None else directory
    found: dict[Path, None] = {}
    for pattern in LIBRARY_GLOBS:
        for path in sorted(directory.glob(pattern)):
            found.setdefault(path.resolve(), None)
    return list(found)


class Library:
    """The process's ``relm_mp`` library: loaded and vetted at most once."""

    def __init__(self, torch_module=None, candidates=None) -> None:
        self._torch = torch_module
        self._candidates = candidates
        self._lock = threading.Lock()
        self.path: Path | None = None
        self.info: BuildInfo | None = None
        self.error: Exception | None = None
        self._done = False

    def _t(self):
        t = self._torch if self._torch is not None else torch
        if t is None:
            raise ModuleNotFoundError("relmo_b200.ops.mp requires torch.") from TORCH_IMPORT_ERROR
        return t

    def _load(self) -> None:
        t = self._t()
        paths = self._candidates() if self._candidates is not None else candidate_libraries()
        if not paths:
            raise FileNotFoundError(
                "Could not find relm_mp custom op library in the relmo_b200 package directory "
                "(build it with `python -m relmo_b200.build`)."
            )
        failures: list[str] = []
        for path in paths:
            try:
                t.ops.load_library(str(path))
                ns = getattr(t.ops, NAMESPACE, None)
                missing = [op for op in REQUIRED_NAMESPACE_OPS if ns is None or not hasattr(ns, op)]
                if missing:
                    raise RuntimeError(f"torch.ops.{NAMESPACE} lacks {', '.join(missing)}")
            except Exception as exc:
                failures.append(f"{path.name}: {exc}")
                continue
            self.path = path
            self.info = BuildInfo.parse(ns.build_info())
            check_compat(
                self.info, str(t.__version__), cuda_tag_of(getattr(t.version, "cuda", None)),
                Policy.from_env().version_policy,
            )
            return
        raise RuntimeError("Failed to load relm_mp custom op library: " + "; ".join(failures))

    def load(self) -> "Library":
        """Load and vet the library (first call), or re-raise the first failure."""

        if not self._done:
            with self._lock:
                if not self._done:
                    try:
                        self._load()
                    except Exception as exc:
                        self.error = exc
                    self._done = True
        if self.error is not None:
            raise RuntimeError(f"relm_mp library unavailable: {self.error}") from self.error
        return self

    def usable(self) -> bool:
        try:
            self.load()
        except Exception:
            return False
        return True

    def ops(self):
        self.load()
        return getattr(self._t().ops, NAMESPACE)

    def has_op(self, op_name: str) -> bool:
        """Whether the loaded library registers ``op_name`` (in the reference
        namespace or in this package's own, ``OWN_NAMESPACE``)."""

        self.load()
        ops = self._t().ops
        return hasattr(getattr(ops, NAMESPACE), op_name) or hasattr(getattr(ops, OWN_NAMESPACE, None), op_name)


_LIBRARY = Library()


def library() -> Library:
    return _LIBRARY


def ops_namespace():
    """``torch.ops.relm_mp`` of the loaded library."""

    return _LIBRARY.ops()


def assert_runtime_compat() -> dict[str, str]:
    """Load the library if needed; raise if it cannot run here. Returns its build_info fields."""

    require_torch("mp compatibility checks")
    _LIBRARY.load()
    return dict(_LIBRARY.info.fields) if _LIBRARY.info else {}


def available() -> bool:
    """True when the library loads and is compatible with this torch."""

    return torch is not None and _LIBRARY.usable()


def loaded_library_paths() -> list[str]:
    """Shared objects of this package mapped into the process (for reports)."""

    if not sys.platform.startswith("linux"):
        return []
    pkg = str(package_dir())
    seen: dict[str, None] = {}
    try:
        with open("/proc/self/maps") as fh:
            for line in fh:
                path = line.split()[-1] if line.strip() else ""
                if path.startswith(pkg) and path.endswith(".so"):
                    seen.setdefault(path, None)
    except OSError:  # pragma: no cover
        pass
    return list(seen)
