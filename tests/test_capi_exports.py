"""CPU checks of the native library: it loads without a GPU and exports every function that
include/*.h declares (no compute calls are made here)."""

from __future__ import annotations

import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"B200EP_API\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            names.append(m.group(1))
        for m in re.finditer(r"^\s*(?:ORT_EXPORT|B200EP_ORT_EXPORT)\s+[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_functions()
    for required in ("b200ep_matmulnbits", "b200ep_group_query_attention", "b200ep_rms_norm",
                     "b200ep_skip_rms_norm", "b200ep_matmulnbits_dequant"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    from onnxruntime_ep_b200 import library_path

    lib = ctypes.CDLL(library_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"symbols declared in include/*.h but not exported: {missing}"


def test_library_reports_version_and_error_text_without_gpu():
    from onnxruntime_ep_b200 import load_library

    lib = load_library()
    assert lib.b200ep_version() >= 10000
    assert isinstance(lib.b200ep_last_error(), bytes)


def test_registration_fails_loudly_without_plugin_entry_points():
    """ORT's plugin-EP headers are not part of this image, so the library exports no
    CreateEpFactories; the registration helper must refuse with its own error before any attempt to
    hand the library to ONNX Runtime (the reference's helper is python/src/onnxruntime_ep_mlx/
    __init__.py:107-132)."""
    import onnxruntime_ep_b200 as pkg

    if pkg.has_plugin_entry_points():
        pytest.skip("this build exports the plugin-EP entry points")
    with pytest.raises(pkg.PluginEntryPointsMissing, match="CreateEpFactories"):
        pkg.register_execution_provider_library()
