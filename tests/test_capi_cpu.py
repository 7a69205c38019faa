"""CPU checks of the C ABI: the library builds, loads without a GPU and
exports every entry point declared in include/qqt_b200.h; host-side config
packing matches the reference's float32 constants."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            names |= set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(qqt_\w+)\s*\(", text, re.M))
    return names


def test_library_exports_every_declared_symbol():
    import __graft_entry__ as ge
    ge.build()
    from qqt_b200 import _capi
    lib = ctypes.CDLL(_capi.LIB_PATH)
    names = _declared()
    assert len(names) >= 10
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    lib.qqt_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.qqt_version()


def test_config_packing_float32_constants():
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import make_ccfg
    cfg = SimConfig(**scenarios.CFG2)
    c = make_ccfg(cfg, 5632, 1.0)
    assert c.obs_stride == 2368 and c.obs_stride % 8 == 0
    assert c.resolve_rounds == 8 and c.danger_rounds == 8
    assert np.float32(c.step_len) == np.float32(0.3)
    assert np.float32(c.chain_time_rest) == np.float32(1.0 - 0.15)
    assert np.float32(c.pen_speed) == np.float32(2 * 0.15)
    assert np.float32(c.h_minus_rad) == np.float32(13 - 0.3)
    assert c.corridor == 1 and c.combo_on == 1


def test_ctypes_structs_match_the_c_header(tmp_path):
    """The ctypes mirrors of the header's structs have the C compiler's
    field offsets and sizes (gcc on include/qqt_b200.h)."""
    import json
    import shutil
    import subprocess
    from qqt_b200 import _capi
    if shutil.which("gcc") is None:
        import pytest
        pytest.skip("no C compiler")
    structs = {"QqtCfg": _capi.QqtCfg, "QqtState": _capi.QqtState,
               "QqtTemplate": _capi.QqtTemplate, "QqtStepOut": _capi.QqtStepOut,
               "QqtMapGen": _capi.QqtMapGen}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "qqt_b200.h"',
             'int main(void) {', 'printf("{");']
    first = True
    for name, cls in structs.items():
        for f in [f[0] for f in cls._fields_] + ["__size__"]:
            expr = f"sizeof({name})" if f == "__size__" else f"offsetof({name}, {f})"
            sep = "" if first else ","
            first = False
            lines.append(f'printf("{sep}\\"{name}.{f}\\": %zu", (size_t)({expr}));')
    lines += ['printf("}\\n");', "return 0; }"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    c = json.loads(subprocess.run([str(exe)], check=True, capture_output=True,
                                  text=True).stdout)
    for name, cls in structs.items():
        for f in [f[0] for f in cls._fields_]:
            assert getattr(cls, f).offset == c[f"{name}.{f}"], f"{name}.{f}"
        assert ctypes.sizeof(cls) == c[f"{name}.__size__"], name
