"""Where one facade call runs: the library's op, or the Python formulas.

The rule, for tensors on a device D:

* D is CUDA: always the library. When it is disabled (``RELM_MP_ENABLE=0``) or
  unusable, the call raises: there is no GPU fallback, so a GPU result always
  comes from the B200 kernels. (relmo fell back to its Python formulas here.)
* D is the CPU: the library's CPU kernels when it is enabled and usable, as
  relmo sends CPU tensors to its library. Otherwise the Python formulas
  (``mp_pack``, ``mp_lgan``), or, under ``RELM_MP_FALLBACK=error``, a
  RuntimeError. A library that lacks the op (an op this package does not
  build) also sends the call to the formulas, as relmo's ``namespace_has_op``
  check does.
"""

from __future__ import annotations

from .mp_runtime import Policy, library

CUSTOM = "custom"
PYTHON = "python"


def is_cuda(tensor: object) -> bool:
    return bool(getattr(tensor, "is_cuda", False))


def _has_op(op_name: str) -> bool:
    return library().has_op(op_name)


def route(op_name: str, tensor: object) -> str:
    """CUSTOM or PYTHON for a call of ``op_name`` whose data lives where ``tensor`` does."""

    policy = Policy.from_env()
    if is_cuda(tensor):
        if not policy.enabled:
            raise RuntimeError(
                f"{op_name}: RELM_MP_ENABLE=0 but relmo_b200 has no GPU fallback; CUDA tensors always run "
                "the B200 kernels."
            )
        try:
            library().load()
        except Exception as exc:
            raise RuntimeError(f"Custom mp op {op_name} is unavailable for CUDA tensors (no GPU fallback).") from exc
        if not _has_op(op_name):
            raise RuntimeError(f"Custom mp op {op_name} is not in the loaded relm_mp library (no GPU fallback).")
        return CUSTOM
    if not policy.enabled:
        return PYTHON
    try:
        library().load()
        if _has_op(op_name):
            return CUSTOM
        reason: Exception | None = None
    except Exception as exc:
        reason = exc
    if policy.on_unavailable == "error":
        raise RuntimeError(f"Custom mp op {op_name} is unavailable.") from reason
    return PYTHON


def call(op_name: str, *args, tensor: object, python):
    """Run ``torch.ops.relm_mp.<op_name>(*args)`` or ``python(*args)`` by :func:`route`."""

    if route(op_name, tensor) == CUSTOM:
        return getattr(library().ops(), op_name)(*args)
    return python(*args)
