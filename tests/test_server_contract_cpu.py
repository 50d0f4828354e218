"""The reference's HTTP server against this package's model and scheduler.

``server.py`` (the reference's FastAPI front end) is kept unchanged on top of
the new path: it imports ``ModelConfig``, ``Model`` and ``load_weights`` from
the model module and ``EOS_TOKEN_IDS``, ``Request`` and ``Scheduler`` from the
scheduler module, builds the engine in ``init_engine`` and drives requests
through ``submit_request`` and each request's asyncio ``token_queue``. These
tests read the reference's own ``server.py`` (where a checkout of the
reference is present; skipped elsewhere) and check every name it imports,
every call it makes into the two modules and every request attribute it
reads against ``mi_b200.model`` / ``mi_b200.scheduler``; and that
``ModelConfig.from_pretrained`` reads a HuggingFace ``config.json`` as the
reference's does. The request flow itself runs on a GPU in
``tests/test_server_flow_gpu.py``.
"""
import ast
import dataclasses
import inspect
import json
import os
import sys

import pytest

REF = os.environ.get("MI_REFERENCE_DIR", "/root/reference")
SERVER = os.path.join(REF, "server.py")
pytestmark = pytest.mark.skipif(not os.path.exists(SERVER),
                                reason="no checkout of the reference here")


def _tree():
    with open(SERVER) as f:
        return ast.parse(f.read())


def _modules():
    from mi_b200 import model, scheduler
    return {"model": model, "scheduler": scheduler}


def test_every_imported_name_exists():
    mods = _modules()
    seen = 0
    for node in ast.walk(_tree()):
        if isinstance(node, ast.ImportFrom) and node.module in mods:
            for alias in node.names:
                assert hasattr(mods[node.module], alias.name), (node.module, alias.name)
                seen += 1
    assert seen >= 6


def _calls(name):
    for node in ast.walk(_tree()):
        if isinstance(node, ast.Call):
            f = node.func
            fname = f.id if isinstance(f, ast.Name) else (f.attr if isinstance(f, ast.Attribute)
                                                          else None)
            if fname == name:
                yield node


def _bind(target, call, skip_self=False):
    """Bind the call's positional count and keyword names to ``target``'s signature."""
    sig = inspect.signature(target)
    params = list(sig.parameters.values())[1:] if skip_self else list(sig.parameters.values())
    sig = sig.replace(parameters=params)
    args = [object()] * len(call.args)
    kwargs = {k.arg: object() for k in call.keywords if k.arg is not None}
    sig.bind(*args, **kwargs)


def test_every_call_into_the_modules_binds():
    from mi_b200.model import Model, ModelConfig, load_weights
    from mi_b200.scheduler import Request, Scheduler
    targets = {"Scheduler": (Scheduler.__init__, True), "Request": (Request, False),
               "load_weights": (load_weights, False), "Model": (Model.__init__, True),
               "from_pretrained": (ModelConfig.from_pretrained, False)}
    bound = {}
    for name, (target, skip) in targets.items():
        for call in _calls(name):
            _bind(target, call, skip)
            bound[name] = bound.get(name, 0) + 1
    assert set(bound) == set(targets), bound
    # the engine methods server.py calls
    for meth in ("start", "submit_request"):
        assert callable(getattr(Scheduler, meth))


def test_request_attributes_server_reads_exist():
    from mi_b200.scheduler import Request
    fields = {f.name for f in dataclasses.fields(Request)}
    used = set()
    for node in ast.walk(_tree()):
        if (isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name)
                and node.value.id == "req"):
            used.add(node.attr)
    assert used and used <= fields, used - fields
    assert {"token_queue", "finish_reason"} <= used


def test_from_pretrained_reads_a_config_like_the_reference(tmp_path):
    sys.path.insert(0, REF)
    try:
        import model as ref_model
    finally:
        sys.path.remove(REF)
    from mi_b200.model import ModelConfig
    cfg = {"hidden_size": 896, "num_attention_heads": 14, "num_key_value_heads": 2,
           "num_hidden_layers": 24, "intermediate_size": 4864, "vocab_size": 151936,
           "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "max_position_embeddings": 32768,
           "tie_word_embeddings": True, "model_type": "qwen2"}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    ours = ModelConfig.from_pretrained(str(tmp_path))
    theirs = ref_model.ModelConfig.from_pretrained(str(tmp_path))
    for f in dataclasses.fields(theirs):
        assert getattr(ours, f.name) == getattr(theirs, f.name), f.name
