"""Import alias for the framework package.

The package lives in the directory ``rl_cs1.6_surf_b200/``; a dot is not
legal in a Python module name, so this module loads that directory as the
package ``surfb200`` (``import surfb200``, ``from surfb200.sim import ...``).
"""
import importlib.util as _ilu
import os as _os
import sys as _sys

_dir = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "rl_cs1.6_surf_b200")
_spec = _ilu.spec_from_file_location("surfb200", _os.path.join(_dir, "__init__.py"),
                                     submodule_search_locations=[_dir])
_mod = _ilu.module_from_spec(_spec)
_sys.modules["surfb200"] = _mod
_spec.loader.exec_module(_mod)

if __name__ == "__main__":      # python -m surfb200 <command> ...
    from surfb200.cli import main as _main
    _sys.exit(_main())
