"""Every name the reference's harnesses import from the modules that the
drop-ins replace exists in the drop-in of that name, and every keyword argument
those harnesses pass at a call site is accepted (CPU only: signatures are
bound, nothing is launched). The fixture ``golden/dropin_api.json`` lists the
imports and keywords, read from the reference's sources by
``golden/make_dropin_api.py``; with it a reference harness such as the
capacity-gate sweep runs unchanged with ``cache-barrier_b200/dropin`` first on
``sys.path``."""

import importlib
import inspect
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
API = json.load(open(os.path.join(HERE, "golden", "dropin_api.json")))


def _target(obj):
    """The callable whose signature a call site binds: a kernel launcher's
    ``kernel[grid](...)`` binds the object ``kernel[grid]`` returns."""
    if hasattr(obj, "__getitem__") and not callable(obj):
        return obj[(1,)]
    return obj


def test_fixture_covers_the_gate_and_carm_harnesses():
    imp = API["imports"]
    assert {"kernel_batched_w4a16_simple", "quantize_weights_int4", "batched_int4_gemm"} <= set(imp["bench_l2_barrier"])
    assert {"quantize_weights_w8", "quantize_acts_w8", "w8a8_bmm", "_pick_config"} <= set(imp["w8a8_bmm"])


@pytest.mark.parametrize("module", sorted(API["imports"]))
def test_every_imported_name_exists(module):
    mod = importlib.import_module(module)
    missing = [n for n in API["imports"][module] if not hasattr(mod, n)]
    assert not missing, f"{module} lacks {missing} (imported by {[API['imports'][module][n] for n in missing]})"


@pytest.mark.parametrize("name", sorted(n for n, ks in API["call_keywords"].items() if ks))
def test_call_site_keywords_are_accepted(name):
    owner = next(m for m, names in API["imports"].items() if name in names)
    fn = _target(getattr(importlib.import_module(owner), name))
    sig = inspect.signature(fn)
    params = sig.parameters
    takes_var_kw = any(p.kind == inspect.Parameter.VAR_KEYWORD for p in params.values())
    for kw in API["call_keywords"][name]:
        assert kw in params or takes_var_kw, f"{owner}.{name} does not accept keyword {kw}"
