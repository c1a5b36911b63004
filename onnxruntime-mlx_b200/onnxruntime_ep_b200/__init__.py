"""onnxruntime_ep_b200: locator and bindings for the B200 int4 decode execution provider.

Mirrors the reference's Python package (python/src/onnxruntime_ep_mlx/__init__.py:1-166): the
same helper names and meaning — ``EP_NAME``, ``ep_name``, ``version``, ``vendor``,
``library_path``, ``register_execution_provider_library``, ``append_to_session_options`` — for
the sm_100a plugin library ``libb200ep.so`` that sits next to this file.  Typical use with an
ONNX Runtime >= 1.29 build::

    import onnxruntime as ort
    import onnxruntime_ep_b200

    onnxruntime_ep_b200.register_execution_provider_library()
    sess = ort.InferenceSession(model, providers=["B200ExecutionProvider", "CPUExecutionProvider"])

``load_library()`` returns the ctypes handle used by the kernel-level bindings in ``ops`` and
the EP-core bindings in ``ep``.
"""

from __future__ import annotations

import ctypes
import os
from typing import Any

__all__ = [
    "EP_NAME",
    "ep_name",
    "version",
    "vendor",
    "library_path",
    "load_library",
    "register_execution_provider_library",
    "append_to_session_options",
    "B200EPError",
    "PluginEntryPointsMissing",
    "has_plugin_entry_points",
    "__version__",
]

#: Name the factory reports to ONNX Runtime.  "MLXExecutionProvider" may be passed as the
#: registration name instead so that applications written for the reference keep their
#: provider lists.
EP_NAME: str = "B200ExecutionProvider"
_VENDOR: str = "onnxruntime-mlx_b200"
_LIB_NAME: str = "libb200ep.so"
__version__: str = "0.1.0"

_lib = None


class B200EPError(RuntimeError):
    """A non-zero status from the native library (message from b200ep_last_error)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


def ep_name() -> str:
    return EP_NAME


def version() -> str:
    return __version__


def vendor() -> str:
    return _VENDOR


def library_path() -> str:
    """Absolute path of the bundled ``libb200ep.so``; FileNotFoundError when it was not built."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)
    if not os.path.isfile(path):
        raise FileNotFoundError(
            f"B200 EP library not found at {path!r}; build it with "
            "`python onnxruntime-mlx_b200/build.py`."
        )
    return path


def load_library() -> ctypes.CDLL:
    """Load libb200ep.so once per process (raises if it is missing — there is no fallback)."""
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(library_path(), mode=ctypes.RTLD_GLOBAL)
        lib.b200ep_last_error.restype = ctypes.c_char_p
        lib.b200ep_version.restype = ctypes.c_int
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = load_library().b200ep_last_error()
        raise B200EPError(status, msg.decode() if msg else "")


def _import_onnxruntime():
    try:
        import onnxruntime as ort  # type: ignore
    except ImportError as exc:  # pragma: no cover - depends on the environment
        raise ImportError("onnxruntime>=1.29 is required to register the B200 execution provider") from exc
    return ort


class PluginEntryPointsMissing(RuntimeError):
    """The library was built without ONNX Runtime's plugin-EP entry points (CreateEpFactories /
    ReleaseEpFactory), so ONNX Runtime cannot load it as an execution provider."""


def has_plugin_entry_points() -> bool:
    """Whether libb200ep.so exports ONNX Runtime's plugin-EP factory functions.  They are compiled
    only against ONNX Runtime's own EP C API headers (onnxruntime_ep_c_api.h, ORT >= 1.29); a build
    without those headers exports the neutral C ABI of b200ep.h / b200ep_ep.h only."""
    lib = load_library()
    return all(hasattr(lib, sym) for sym in ("CreateEpFactories", "ReleaseEpFactory"))


def register_execution_provider_library(name: str = EP_NAME) -> str:
    """Register libb200ep.so with ONNX Runtime under ``name``; returns the library path.

    Raises PluginEntryPointsMissing when the library has no CreateEpFactories (built without ONNX
    Runtime's EP headers) — before onnxruntime is asked to load it — and ImportError when
    onnxruntime itself is not installed."""
    if not has_plugin_entry_points():
        raise PluginEntryPointsMissing(
            "libb200ep.so was built without ONNX Runtime's plugin-EP entry points (CreateEpFactories / "
            "ReleaseEpFactory): the EP core is reachable through the C ABI of b200ep_ep.h "
            "(onnxruntime_ep_b200.ep), but ONNX Runtime cannot load this build as an execution provider")
    ort = _import_onnxruntime()
    if not hasattr(ort, "register_execution_provider_library"):
        raise RuntimeError("this onnxruntime has no register_execution_provider_library (needs >= 1.29)")
    lib = library_path()
    ort.register_execution_provider_library(name, lib)
    return lib


def append_to_session_options(session_options: Any, name: str = EP_NAME,
                              provider_options: "dict[str, str] | None" = None) -> Any:
    register_execution_provider_library(name)
    if not hasattr(session_options, "add_provider"):
        raise RuntimeError(
            "this onnxruntime build has no SessionOptions.add_provider; pass "
            f'providers=["{name}", "CPUExecutionProvider"] to InferenceSession instead')
    session_options.add_provider(name, dict(provider_options or {}))
    return session_options
