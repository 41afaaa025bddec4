"""The SGLang MoE-method hook (reference PATCH:450-581) without SGLang: a fake
``sglang`` module tree stands in for the classes the hook touches, and the
two ops it calls are replaced by recorders, so only the hook's own logic runs
(wiring, argument plumbing, refusals).  Runs on CPU."""

import sys
import types

import pytest
import torch

import dsv4_b200.sglang_hook as H


class _Method:
    def __init__(self, config):
        self.runner = types.SimpleNamespace(config=config)
        self.prefix = "model.layers.3.mlp.experts"

    def process_weights_after_loading(self, layer):
        raise AssertionError("original should be replaced")

    def apply(self, layer, dispatch_output):
        return "original"


@pytest.fixture
def fake_sglang(monkeypatch):
    class StandardCombineInput:
        def __init__(self, hidden_states):
            self.hidden_states = hidden_states

    class TopKOutputChecker:
        @staticmethod
        def format_is_standard(topk_output):
            return topk_output.format == "standard"

    mods = {}
    for name in ["sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.quantization",
                 "sglang.srt.layers.quantization.mxfp4_marlin_moe", "sglang.srt.layers.moe",
                 "sglang.srt.layers.moe.topk", "sglang.srt.layers.moe.token_dispatcher",
                 "sglang.srt.layers.moe.token_dispatcher.standard"]:
        mods[name] = types.ModuleType(name)
        monkeypatch.setitem(sys.modules, name, mods[name])
    mods["sglang.srt.layers.quantization"].mxfp4_marlin_moe = mods[
        "sglang.srt.layers.quantization.mxfp4_marlin_moe"]
    mods["sglang.srt.layers.quantization.mxfp4_marlin_moe"].Mxfp4MarlinMoEMethod = _Method
    mods["sglang.srt.layers.moe.topk"].TopKOutputChecker = TopKOutputChecker
    mods["sglang.srt.layers.moe.token_dispatcher.standard"].StandardCombineInput = StandardCombineInput
    saved = {k: _Method.__dict__[k] for k in ("apply", "process_weights_after_loading")}
    yield types.SimpleNamespace(StandardCombineInput=StandardCombineInput)
    for k, v in saved.items():
        setattr(_Method, k, v)
    if hasattr(_Method, "_sglang_original_apply"):
        del _Method._sglang_original_apply


@pytest.fixture
def recorders(monkeypatch):
    calls = {}

    def prepare(layer, *, headroom_bits, topk):
        calls["prepare"] = dict(layer=layer, headroom_bits=headroom_bits, topk=topk)
        w2_mxfp4 = torch.zeros((4, 64 // 32, 16, 128), dtype=torch.uint8)  # I = 64
        layer._dsv4_mxfp4_int8_weights = types.SimpleNamespace(
            w2_mxfp4=w2_mxfp4, w2_channel_scale=torch.zeros((4, 128)))  # H = 128

    def forward(**kw):
        calls["forward"] = kw
        return torch.full_like(kw["hidden_states"], 7.0)

    monkeypatch.setattr(H, "prepare_mxfp4_int8_moe", prepare)
    monkeypatch.setattr(H, "mxfp4_int8_moe_forward", forward)
    return calls


def _layer():
    layer = torch.nn.Module()
    layer.w13_weight = torch.nn.Parameter(torch.zeros((4, 128, 64), dtype=torch.uint8),
                                          requires_grad=False)
    layer.w2_weight = torch.nn.Parameter(torch.zeros((4, 128, 32), dtype=torch.uint8),
                                         requires_grad=False)
    return layer


def _cfg(**kw):
    base = dict(num_experts_per_tok=8, routed_scaling_factor=2.5, swiglu_limit=10.0,
                apply_router_weight_on_input=False)
    base.update(kw)
    return types.SimpleNamespace(**base)


def test_install_process_and_apply(fake_sglang, recorders, monkeypatch):
    monkeypatch.setenv("SGLANG_DSV4_MXFP4_INT8_HEADROOM_BITS", "2")
    cls = H.install()
    assert cls is _Method and _Method._sglang_original_apply is not None
    assert _Method.apply is H.apply and _Method.process_weights_after_loading is H.process_weights_after_loading
    H.install()  # idempotent: the original stays the original
    assert _Method._sglang_original_apply(None, None, None) == "original"

    method, layer = _Method(_cfg()), _layer()
    method.process_weights_after_loading(layer)
    assert layer.w13_weight.dtype == torch.int8 and layer.w2_weight.dtype == torch.int8
    assert recorders["prepare"]["topk"] == 8 and recorders["prepare"]["headroom_bits"] == 2
    assert layer._dsv4_mxfp4_backend == H.BACKEND_TAG

    hidden = torch.randn(5, 128)
    topk = types.SimpleNamespace(format="standard", topk_ids=torch.zeros((5, 8), dtype=torch.int32),
                                 topk_weights=torch.ones((5, 8)))
    out = method.apply(layer, types.SimpleNamespace(hidden_states=hidden, topk_output=topk))
    assert isinstance(out, fake_sglang.StandardCombineInput)
    assert torch.equal(out.hidden_states, torch.full_like(hidden, 7.0))
    kw = recorders["forward"]
    assert kw["hidden_size"] == 128 and kw["intermediate_size"] == 64
    assert kw["routed_scaling_factor"] == 2.5 and kw["clamp_limit"] == 10.0
    assert kw["apply_router_weight_on_input"] is False
    assert kw["topk_ids"] is topk.topk_ids and kw["topk_weights"] is topk.topk_weights


def test_refusals(fake_sglang, recorders, monkeypatch):
    H.install()
    method, layer = _Method(_cfg()), _layer()
    topk = types.SimpleNamespace(format="standard", topk_ids=None, topk_weights=None)
    with pytest.raises(RuntimeError, match="not prepared"):
        method.apply(layer, types.SimpleNamespace(hidden_states=torch.zeros(1, 128), topk_output=topk))
    method.process_weights_after_loading(layer)
    bad = types.SimpleNamespace(format="triton_kernel", topk_ids=None, topk_weights=None)
    with pytest.raises(ValueError, match="topk output format"):
        method.apply(layer, types.SimpleNamespace(hidden_states=torch.zeros(1, 128), topk_output=bad))
    mega = _layer()
    mega._mega_moe_weights_built = True
    with pytest.raises(RuntimeError, match="MegaMoE"):
        method.process_weights_after_loading(mega)
    monkeypatch.setenv("SGLANG_DSV4_MXFP4_MOE_BACKEND", "ogs")
    with pytest.raises(ValueError, match="OGS"):
        method.process_weights_after_loading(_layer())


def test_without_sglang_returns_plain_combine_input(recorders):
    layer = _layer()
    H.process_weights_after_loading(types.SimpleNamespace(), layer)
    assert recorders["prepare"]["topk"] is None
    topk = types.SimpleNamespace(topk_ids=None, topk_weights=None)
    out = H.apply(types.SimpleNamespace(), layer,
                  types.SimpleNamespace(hidden_states=torch.zeros(2, 128), topk_output=topk))
    assert isinstance(out, H.CombineInput)
    assert recorders["forward"]["routed_scaling_factor"] is None
    with pytest.raises(ImportError):
        H.install()
