"""Write tests/golden/pinfer_py_bindings.json: the ctypes binding table of the reference's own
Python package (python/pinfer/_lib.py: the required table, the feature-detected optional table,
and the layouts of the structs passed by pointer), as that package binds them when it loads a
library. tests/test_gpu_dropin.py binds this repository's library from the recorded table and
runs the package's call sequence on the device, so the drop-in is checked where the reference
checkout is absent.

    NB_REFERENCE=<checkout> python tests/golden/make_pinfer_py_bindings.py

Needs the reference checkout (its python/ package is imported) and a built
nibblemac_b200/lib/libpinfer.so (the package only binds against a loaded library).
"""
from __future__ import annotations

import ctypes
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def type_name(t) -> str | None:
    if t is None:
        return None
    if hasattr(t, "_type_") and isinstance(t._type_, type) and issubclass(t, ctypes._Pointer):
        return "POINTER(" + type_name(t._type_) + ")"
    if hasattr(t, "_argtypes_"):   # a CFUNCTYPE
        return "CFUNC(" + ",".join(type_name(a) for a in (t._restype_, *t._argtypes_)) + ")"
    return t.__name__


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else
               os.environ.get("NB_REFERENCE", ROOT.parent / "reference"))
    sys.path.insert(0, str(ref / "python"))
    from pinfer import _lib
    lib = _lib.load_library(ROOT / "nibblemac_b200" / "lib" / "libpinfer.so")
    funcs = {}
    for name in sorted(dir(lib)):
        fn = getattr(lib, name)
        if name.startswith("pinfer_") and fn is not None and hasattr(fn, "argtypes"):
            funcs[name] = {"restype": type_name(fn.restype),
                           "argtypes": [type_name(a) for a in (fn.argtypes or [])],
                           "required": name in _lib._REQUIRED}
    structs = {}
    for cls in (_lib.Params, _lib.SpecParams, _lib.SpecStats, _lib.GenOpts):
        structs[cls.__name__] = {"size": ctypes.sizeof(cls),
                                 "fields": [[f[0], type_name(f[1]), getattr(cls, f[0]).offset]
                                            for f in cls._fields_]}
    out = Path(__file__).with_name("pinfer_py_bindings.json")
    out.write_text(json.dumps({"about": "ctypes bindings of the reference package python/pinfer/_lib.py",
                               "functions": funcs, "structs": structs}, indent=1) + "\n")
    print(f"wrote {out}: {len(funcs)} functions")


if __name__ == "__main__":
    main()
