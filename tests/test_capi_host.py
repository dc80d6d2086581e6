"""C ABI and host-side logic on the CPU: the library loads without a GPU, exports
every symbol ``include/gemq_b200.h`` declares, and rejects bad arguments with the
documented status before touching the device. Block guards mirror the
reference's truth tables (tests/test_moe_block_equiv.py:255-332 of RobustGEMQ)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "gemq_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(gemq_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from robustgemq_b200 import _lib

    lib = _lib.load()
    declared = header_functions()
    assert len(declared) >= 18
    assert sorted(_lib.EXPORTED) == declared
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.gemq_version() == 1


def _fake_proj(E=2, K=128, N=128, g=64):
    from robustgemq_b200._lib import ProjT

    p = ProjT()
    p.wq = p.scales = p.zeros = p.nbits = p.wq_strides = p.zs_strides = 0x1000
    p.wq_rows, p.num_experts, p.k, p.n, p.group_size = 64, E, K, N, g
    return p


def _status(rc):
    from robustgemq_b200 import _lib

    return rc, _lib.load().gemq_last_error_string().decode()


def test_argument_errors_are_statuses_not_aborts():
    from robustgemq_b200 import _lib

    lib = _lib.load()
    rc, msg = _status(lib.gemq_pack_weights_over_cols(None, 4, 8, 5, None, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT and "bitwidth" in msg
    rc, _ = _status(lib.gemq_unpack_over_cols(None, 4, 1, 64, 2, None, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT  # 64 two-bit codes need 4 words, 1 given
    p = _fake_proj()
    p.k = 100  # not a multiple of group_size
    rc, msg = _status(lib.gemq_dequant_expert(ctypes.byref(p), 0, 0x2000, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT and "group_size" in msg
    p = _fake_proj()
    rc, _ = _status(lib.gemq_dequant_expert(ctypes.byref(p), 5, 0x2000, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT
    rc, _ = _status(lib.gemq_dequant_group_gemm(ctypes.byref(p), 0x3000, 4, 0x4000, 0, 0x5000, 0x6000, 1 << 20, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT  # no indices
    rc, _ = _status(lib.gemq_dequant_group_gemm(ctypes.byref(p), 0x3000, 4, 0x4000, 1, 0x5000, 0x6000, 8, None))
    assert rc == _lib.GEMQ_ERR_WORKSPACE
    # index a's output rows start at a * m, a 32-bit row offset: 600 x 2^22 rows is too many
    rc, msg = _status(lib.gemq_dequant_group_gemm(ctypes.byref(p), 0x3000, 1 << 22, 0x4000, 600, 0x5000, 0x6000,
                                                  1 << 20, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT and "2^31" in msg


@pytest.mark.parametrize("num_indices,m,x,out,indices,text", [
    (1024, 4, 0x3000, 0x5000, 0x4000, "GEMQ_NOALLOC_MAX_INDICES"),
    (0, 4, 0x3000, 0x5000, 0x4000, "positive"),
    (-1, 4, 0x3000, 0x5000, 0x4000, "positive"),
    (600, 1 << 22, 0x3000, 0x5000, 0x4000, "2^31"),
    (4, 4, None, 0x5000, 0x4000, "null"),
    (4, 4, 0x3000, None, 0x4000, "null"),
    (4, 4, 0x3000, 0x5000, None, "null"),
])
def test_noalloc_group_gemm_rejects_arguments_before_device_access(num_indices, m, x, out, indices, text):
    """The allocation-free entry point checks its arguments on the host: these
    calls get GEMQ_ERR_INVALID_ARGUMENT without a CUDA call (no GPU here)."""
    from robustgemq_b200 import _lib

    lib = _lib.load()
    p = _fake_proj()
    rc, msg = _status(lib.gemq_dequant_group_gemm_noalloc(ctypes.byref(p), x, m, indices, num_indices, out, None))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT
    assert text in msg


def _desc(**kw):
    from robustgemq_b200._lib import LayerDescT

    d = LayerDescT()
    d.hidden, d.inter, d.num_experts, d.top_k, d.group_size = 128, 128, 2, 1, 64
    d.gate_weight = 0x1000
    d.w1, d.w3, d.w2 = _fake_proj(), _fake_proj(), _fake_proj()
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("field,value,text", [
    ("top_k", 3, "top_k"),
    ("num_experts", 300, "256"),
    ("group_size", 128, "Group sizes"),
    ("router", 7, "router"),
    ("gate_weight", None, "gate"),
])
def test_layer_create_validates_before_device_access(field, value, text):
    from robustgemq_b200 import _lib

    lib = _lib.load()
    d = _desc(**{field: value})
    h = ctypes.c_void_p()
    rc, msg = _status(lib.gemq_layer_create(ctypes.byref(d), ctypes.byref(h)))
    assert rc in (_lib.GEMQ_ERR_INVALID_ARGUMENT, _lib.GEMQ_ERR_UNSUPPORTED)
    assert text in msg


def test_layer_shape_mismatch_rejected():
    from robustgemq_b200 import _lib

    lib = _lib.load()
    d = _desc()
    d.w2.n = 256  # down projection must map F -> D
    h = ctypes.c_void_p()
    rc, msg = _status(lib.gemq_layer_create(ctypes.byref(d), ctypes.byref(h)))
    assert rc == _lib.GEMQ_ERR_INVALID_ARGUMENT and "shapes" in msg


def test_workspace_size_queries_grow_with_tokens():
    from robustgemq_b200 import _lib

    lib = _lib.load()
    assert lib.gemq_group_gemm_workspace_size(4) >= lib.gemq_group_gemm_workspace_size(1) > 0
    assert lib.gemq_moe_workspace_size(None, 16, 0) == 0


# ----------------------------------------------------------------------------- guards
def _ds_config(**kw):
    c = SimpleNamespace(hidden_size=64, moe_intermediate_size=64, n_routed_experts=4, n_shared_experts=2,
                        num_experts_per_tok=2, norm_topk_prob=False, topk_method="greedy", scoring_func="softmax",
                        routed_scaling_factor=1.0)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


class _OfficialBlockStub:
    pass


_OfficialBlockStub.__module__ = "transformers_modules.deepseek.modeling_deepseek"


class _BuiltinBlockStub:
    pass


_BuiltinBlockStub.__module__ = "transformers.models.deepseek_v2.modeling_deepseek_v2"


@pytest.mark.parametrize("fields", [
    dict(scoring_func="sigmoid"), dict(topk_method="noaux_tc"),
    dict(topk_method="group_limited_greedy", n_group=3, topk_group=1),   # 3 does not divide 4 experts
    dict(topk_method="group_limited_greedy", n_group=2, topk_group=3),   # more kept groups than groups
    dict(topk_method="group_limited_greedy", n_group=4, topk_group=1),   # 1 kept expert < top_k = 2
])
def test_deepseek_feature_guard(fields):
    from robustgemq_b200.inference import check_deepseek_routing_supported, deepseek_group_routing

    check_deepseek_routing_supported(_ds_config())
    ok = _ds_config(topk_method="group_limited_greedy", n_group=2, topk_group=1)
    check_deepseek_routing_supported(ok)
    assert deepseek_group_routing(ok) == (2, 1)
    assert deepseek_group_routing(_ds_config(n_group=2, topk_group=1)) == (1, 1)  # greedy ignores the groups
    with pytest.raises(AssertionError):
        check_deepseek_routing_supported(_ds_config(**fields))


# (official gate?, norm_topk_prob, top_k, routed_scaling_factor) -> (renormalise, scale) of the
# replaced gate (moe_block.py:31-42 states both rules); the reference's fused block accepts only
# the rows whose rule is (norm_topk_prob, 1.0).
@pytest.mark.parametrize("official,norm,top_k,scaling,rule", [
    (True, False, 2, 1.0, (False, 1.0)), (True, False, 2, 16.0, (False, 16.0)), (True, True, 2, 16.0, (True, 1.0)),
    (True, True, 1, 2.0, (False, 2.0)), (False, False, 2, 1.0, (False, 1.0)), (False, True, 2, 1.0, (False, 1.0)),
    (False, False, 2, 16.0, (False, 16.0)),
])
def test_deepseek_gate_rule_table(official, norm, top_k, scaling, rule):
    from robustgemq_b200.inference import check_deepseek_gate_matches

    cfg = _ds_config(norm_topk_prob=norm, num_experts_per_tok=top_k, routed_scaling_factor=scaling)
    blk = _OfficialBlockStub() if official else _BuiltinBlockStub()
    assert check_deepseek_gate_matches(cfg, blk) == rule


@pytest.mark.parametrize("n_group,topk_group,scale", [(3, 1, 1.0), (0, 1, 1.0), (33, 1, 1.0), (4, 5, 1.0),
                                                      (8, 1, 1.0), (4, 2, float("inf")), (4, 2, float("nan"))])
def test_route_ex_rejects_bad_routing_options(n_group, topk_group, scale):
    """Option checks run before any device work (E = 64, k = 16: 8 groups keeping 1 hold
    only 8 experts)."""
    from robustgemq_b200 import _lib

    lib = _lib.load()
    r = _lib.RoutingT(0, n_group, topk_group, scale)
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: the options fail first
    rc = lib.gemq_route_ex(fake, 4, 64, fake, 64, 16, _lib.GEMQ_ROUTER_FP32, ctypes.byref(r), 0, fake, fake, fake,
                           fake, 1 << 16, None)
    assert rc != 0
    assert lib.gemq_layer_set_routing(None, ctypes.byref(r)) != 0


def test_from_hf_requires_packed_linears():
    import torch

    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock

    cfg = SimpleNamespace(hidden_size=64, intermediate_size=64, num_experts=2, num_experts_per_tok=1,
                          norm_topk_prob=False)
    hf = SimpleNamespace(gate=torch.nn.Linear(64, 2, bias=False),
                         experts=[SimpleNamespace(gate_proj=torch.nn.Linear(64, 64), up_proj=None, down_proj=None)])
    with pytest.raises(ValueError, match="patch and replace"):
        QuantFusedOlmoeMoEBlock.from_hf(cfg, hf)


def test_stacking_matches_reference_layout():
    """from_packed stacks like from_hf (moe_block.py:725-757): cat along rows,
    exclusive-cumsum numel strides, one group size, w1/w3 aligned."""
    import torch

    from oracle import gemq_oracle as O
    from robustgemq_b200.inference import QuantFusedOlmoeMoEBlock
    from robustgemq_b200.quant import PackedLinear

    rng = np.random.default_rng(0)
    bits, K, N, g = [2, 3, 4], 128, 64, 64

    def lin(b, k, n):
        codes = rng.integers(0, 2 ** b, size=(n, k), dtype=np.uint8)
        wq = np.ascontiguousarray(O.pack_weights_over_cols(codes, b))
        return PackedLinear(torch.from_numpy(wq), torch.zeros((k // g, n), dtype=torch.float16),
                            torch.zeros((k // g, n), dtype=torch.float16), b, g, k, n)

    cfg = SimpleNamespace(hidden_size=K, intermediate_size=N, num_experts=3, num_experts_per_tok=2,
                          norm_topk_prob=False)
    w1 = [lin(b, K, N) for b in bits]
    w3 = [lin(b, K, N) for b in bits]
    w2 = [lin(b, N, K) for b in bits]
    blk = QuantFusedOlmoeMoEBlock.from_packed(cfg, torch.zeros((3, K), dtype=torch.float16), w1, w3, w2)
    assert blk.block_group_size == g
    assert blk.w1_wq.shape == (sum(O.packed_rows(K, b) for b in bits), N)
    assert blk.w1_wq_strides.tolist() == [0, O.packed_rows(K, 2) * N, (O.packed_rows(K, 2) + O.packed_rows(K, 3)) * N]
    assert blk.w2_zs_strides.tolist() == [0, (N // g) * K, 2 * (N // g) * K]
    bad = [lin(2, K, N), lin(2, K, N), lin(2, K, N)]
    bad[1].group_size = 128
    with pytest.raises(AssertionError, match="Group sizes"):
        QuantFusedOlmoeMoEBlock.from_packed(cfg, torch.zeros((3, K), dtype=torch.float16), bad, bad, w2)


class _FakeCudaTensor:
    """Stands for a CUDA tensor on device ``index`` (this machine has no GPU)."""

    is_cuda = True

    def __init__(self, index):
        self.device = SimpleNamespace(type="cuda", index=index)


def test_calls_switch_to_the_inputs_device(monkeypatch):
    """A model spread over several GPUs in one process calls each layer with its
    inputs on that layer's GPU while another device is current; the Python entry
    points make the input's device current for the call, and only then."""
    import contextlib

    import torch
    from robustgemq_b200 import _lib

    current = {"dev": 0}
    entered = []

    @contextlib.contextmanager
    def fake_device(d):
        entered.append(d.index)
        prev, current["dev"] = current["dev"], d.index
        try:
            yield
        finally:
            current["dev"] = prev

    monkeypatch.setattr(torch.cuda, "current_device", lambda: current["dev"])
    monkeypatch.setattr(torch.cuda, "device", fake_device)
    monkeypatch.setattr(torch, "Tensor", _FakeCudaTensor)  # isinstance check in the decorator

    seen = []

    @_lib.on_input_device
    def op(x, scale=1):
        seen.append(current["dev"])
        return scale

    assert op(_FakeCudaTensor(0)) == 1 and entered == [] and seen == [0]
    assert op(_FakeCudaTensor(1), scale=2) == 2 and entered == [1] and seen == [0, 1]
    assert op(x=_FakeCudaTensor(1)) == 1 and entered == [1, 1] and seen == [0, 1, 1]
    assert current["dev"] == 0  # restored after each call
    assert not _lib.off_current_device(_FakeCudaTensor(0))
    assert _lib.off_current_device(_FakeCudaTensor(3))


def test_header_constants_match_the_python_binding():
    """Every status, router, forward-flag and size constant of include/gemq_b200.h has
    the same value in robustgemq_b200._lib (flags by name without the GEMQ_ prefix)."""
    from robustgemq_b200 import _lib

    header = (Path(__file__).resolve().parents[1] / "include" / "gemq_b200.h").read_text()
    defs = dict(re.findall(r"^#define (GEMQ_[A-Z0-9_]+) (\d+)u?\b", header, flags=re.M))
    assert len(defs) > 20
    for name, value in defs.items():
        if name.startswith("GEMQ_STAGE_") or name in ("GEMQ_NUM_STAGES", "GEMQ_NOALLOC_MAX_INDICES"):
            continue
        py = getattr(_lib, name, None)
        if py is None:
            py = getattr(_lib, name[len("GEMQ_"):], None)
        assert py is not None, name
        assert int(py) == int(value), name
    stages = sorted((int(v), n[len("GEMQ_STAGE_"):].lower()) for n, v in defs.items() if n.startswith("GEMQ_STAGE_"))
    assert tuple(n for _, n in stages) == _lib.STAGES
    assert int(defs["GEMQ_NUM_STAGES"]) == len(_lib.STAGES)
