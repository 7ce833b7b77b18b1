"""Import tests/golden/make_golden.py's seeded-state helpers without running it."""
import importlib.util
import os

_p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "make_golden.py")
_spec = importlib.util.spec_from_file_location("make_golden", _p)
_m = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_m)
gqa_long_cache = _m.gqa_long_cache
gdn_init_state = _m.gdn_init_state
