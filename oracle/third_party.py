"""Include directories of the two header-only libraries the reference's
engine sources need (nlohmann/json for QwenConfig::from_json and the
safetensors header, spdlog for its logging), which the reference does not
vendor.  TEST INFRASTRUCTURE ONLY: used to build the reference engine for the
greedy-token goldens and the CudaBackend drop-in engine test.

Copies shipped inside installed Python packages are found under the
interpreter's site-packages; the system include directories are tried last.

    python oracle/third_party.py      # prints JSON_INC=... SPDLOG_INC=... for make
"""
from __future__ import annotations

import os
import site
import sys

# (header that must exist below the directory, candidate directories relative to a site-packages root)
_JSON = ("nlohmann/json.hpp", ("include/cudnn_frontend/thirdparty", "nlohmann_json/include", "include"))
_SPDLOG = ("spdlog/spdlog.h", ("flashinfer/data/spdlog/include", "spdlog/include", "include"))


def _roots() -> list[str]:
    roots = []
    try:
        roots += site.getsitepackages()
    except AttributeError:
        pass
    roots += [p for p in sys.path if p.endswith("site-packages")]
    return list(dict.fromkeys(roots))


def _find(spec) -> str | None:
    header, rels = spec
    for root in _roots():
        for rel in rels:
            d = os.path.join(root, rel)
            if os.path.exists(os.path.join(d, header)):
                return d
    for d in ("/usr/include", "/usr/local/include"):
        if os.path.exists(os.path.join(d, header)):
            return d
    return None


def make_vars() -> list[str]:
    """`JSON_INC=dir SPDLOG_INC=dir` for make, or [] when either is missing."""
    j, s = _find(_JSON), _find(_SPDLOG)
    if not j or not s:
        return []
    return [f"JSON_INC={j}", f"SPDLOG_INC={s}"]


if __name__ == "__main__":
    print(" ".join(make_vars()))
