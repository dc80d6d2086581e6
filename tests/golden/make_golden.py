"""Generate golden vectors by running the reference's own kernels and MoE blocks.

Run from the repository root in a container that has the reference checkout::

    python tests/golden/make_golden.py --reference <path-to-RobustGEMQ>

The reference kernels (``gemq/triton_kernels/*.py``) run on the CPU under
``TRITON_INTERPRET=1``. Autotuned kernels are launched through ``.fn[grid]`` with
fixed block sizes; the host-side glue below reproduces each wrapper's allocation
and grid (cited per wrapper). ``gemq/inference/moe_block.py`` is imported with two
stand-ins for imports that do not resolve here (``gemlite.core.GemLiteLinearTriton``,
only used in an ``isinstance`` check, and transformers' ``DeepseekV2MoE``, only a
type annotation), and its module-level kernel wrappers are pointed at the
interpreted launches.

Every kernel output is recorded twice:

* ``*_interp``: the stock interpreter, whose ``tl.fma`` evaluates ``x*y + z`` in
  numpy float16 (two roundings);
* ``*_gpu``: the interpreter with ``create_fma`` rounding the exact ``x*y + z``
  once, i.e. the ``fma.rn.f16`` that ``tl.fma`` lowers to on NVIDIA GPUs.

Outputs land in ``tests/golden/*.npz`` (inputs included), read by the tests on
any machine; nothing at test time needs the reference checkout.
"""

from __future__ import annotations

import argparse
import contextlib
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import gemq_oracle as O  # noqa: E402


# --------------------------------------------------------------------------- interpreter fma modes
@contextlib.contextmanager
def fma_mode(mode: str):
    """Swap the interpreter's ``create_fma`` for a single-rounding fp16 fma."""
    from triton.runtime import interpreter as I

    orig = I.InterpreterBuilder.create_fma
    if mode == "interp":
        yield
        return

    def create_fma(self, x, y, z):
        xd, yd, zd = x.data, y.data, z.data
        if zd.dtype == np.float16:
            # fp16 values are integer multiples of 2**-24; the dequant fma has an
            # integer-valued x (the code), so x*Y + Z is exact in int64.
            xi = xd.astype(np.float64)
            assert np.all(xi == np.round(xi)) and np.all(np.abs(xi) < 2 ** 16)
            Y = (yd.astype(np.float64) * 2.0 ** 24).astype(np.int64)
            Z = (np.broadcast_to(zd, np.broadcast_shapes(xd.shape, yd.shape, zd.shape)).astype(np.float64)
                 * 2.0 ** 24).astype(np.int64)
            exact = xi.astype(np.int64) * Y + Z
            out = (exact.astype(np.float64) * 2.0 ** -24).astype(np.float16)
            return I.TensorHandle(out, z.dtype.scalar)
        return orig(self, x, y, z)

    I.InterpreterBuilder.create_fma = create_fma
    try:
        yield
    finally:
        I.InterpreterBuilder.create_fma = orig


# --------------------------------------------------------------------------- interpreted wrappers
class Ref:
    def __init__(self, ref_root: str):
        sys.path.insert(0, ref_root)
        from gemq.triton_kernels import utils, dequant_group_gemm, dequant_gemm, dequant_gemv, fused_dequant_bmm
        self.U, self.G, self.DG, self.GV, self.FB = utils, dequant_group_gemm, dequant_gemm, dequant_gemv, fused_dequant_bmm

    def pack(self, codes: torch.Tensor, nbits: int) -> torch.Tensor:
        # utils.py:74-113 is not autotuned; call the wrapper as is.
        out, _ = self.U.pack_weights_over_cols_triton(codes, nbits)
        return out.contiguous()

    def unpack(self, packed: torch.Tensor, nbits: int, ncols: int) -> torch.Tensor:
        return self.U.unpack_over_cols_triton(packed, nbits, 32, ncols)

    def group_gemm(self, x, indices, wq, scales, zeros, nbits, group_sizes, wq_strides, zs_strides):
        # host glue of dequant_group_gemm.py:155-202
        M, K = x.shape
        _, N = wq.shape
        A, = indices.shape
        E, = nbits.shape
        out = torch.empty((A, M, N), dtype=torch.float16)
        num_sm = 4
        self.G.dequant_group_gemm_kernel.fn[(num_sm,)](
            x, wq, out, indices, scales, zeros, nbits, group_sizes, wq_strides, zs_strides,
            M, N, K, A, E, x.stride(0), x.stride(1), wq.stride(0), wq.stride(1),
            out.stride(0), out.stride(1), out.stride(2), scales.stride(0), scales.stride(1),
            NUM_SM=num_sm, BLOCK_SIZE_M=16, BLOCK_SIZE_N=64, BLOCK_SIZE_K=32)
        return out

    def gemm(self, x, wq, scales, zeros, nbits, group_size):
        # host glue of dequant_gemm.py:150-193
        M, K = x.shape
        _, N = wq.shape
        out = torch.empty((M, N), dtype=torch.float16)
        bm, bn, bk = 16, 64, 32
        grid = (((M + bm - 1) // bm) * ((N + bn - 1) // bn),)
        self.DG.dequant_gemm_kernel.fn[grid](
            x, wq, out, scales, zeros, M, N, K, x.stride(0), x.stride(1), wq.stride(0), wq.stride(1),
            out.stride(0), out.stride(1), scales.stride(0), scales.stride(1), nbits, group_size,
            BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk)
        return out

    def splitk_gemv(self, x, wq, scales, zeros, nbits, group_size):
        # host glue of dequant_gemv.py:118-156 (output zeroed as reset_to_zero does)
        M, K = x.shape
        _, N = wq.shape
        out = torch.zeros((M, N), dtype=torch.float16)
        bn, bk = 64, 64
        grid = ((N + bn - 1) // bn, (K + bk - 1) // bk)
        self.GV.dequant_splitk_gemv_kernel.fn[grid](
            x, wq, out, scales, zeros, N, K, x.stride(0), x.stride(1), wq.stride(0), wq.stride(1),
            out.stride(0), out.stride(1), scales.stride(0), scales.stride(1), nbits, group_size,
            BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk)
        return out

    def up_proj(self, x, idx, w1, w3, s1, z1, s3, z3, nbits, w_strides, group_size):
        # host glue of fused_dequant_bmm.py:122-173
        _, K = x.shape
        _, N = w1.shape
        A, = idx.shape
        x1 = torch.empty((1, A * N), dtype=torch.float16)
        x3 = torch.empty((1, A * N), dtype=torch.float16)
        bn, bk = 64, 128
        grid = ((A * N + bn - 1) // bn,)
        self.FB.fused_dequant_up_proj_kernel.fn[grid](
            x, idx, w1, w3, x1, x3, s1, z1, s3, z3, nbits, w_strides, N, K, A,
            x.stride(0), x.stride(1), w1.stride(0), w1.stride(1), x1.stride(0), x1.stride(1),
            s1.stride(0), s1.stride(1), group_size, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk)
        return x1, x3

    def down_proj(self, x1, x3, idx, w2, s2, z2, nbits, w_strides, group_size):
        # host glue of fused_dequant_bmm.py:264-312
        _, AK = x1.shape
        _, N = w2.shape
        A, = idx.shape
        K = AK // A
        x2 = torch.empty((1, A * N), dtype=torch.float16)
        bn, bk = 64, 128
        grid = ((A * N + bn - 1) // bn,)
        self.FB.fused_dequant_down_proj_kernel.fn[grid](
            x1, x3, idx, w2, x2, s2, z2, nbits, w_strides, N, K, A,
            x1.stride(0), x1.stride(1), w2.stride(0), w2.stride(1), x2.stride(0), x2.stride(1),
            s2.stride(0), s2.stride(1), group_size, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk)
        return x2


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def proj_tensors(p: O.PackedProj):
    return (t(p.wq), t(p.scales), t(p.zeros), t(p.nbits), t(p.group_sizes), t(p.wq_strides), t(p.zs_strides))


def proj_arrays(prefix: str, p: O.PackedProj) -> dict:
    return {f"{prefix}_wq": p.wq, f"{prefix}_scales": p.scales, f"{prefix}_zeros": p.zeros,
            f"{prefix}_nbits": p.nbits, f"{prefix}_group_sizes": p.group_sizes,
            f"{prefix}_wq_strides": p.wq_strides, f"{prefix}_zs_strides": p.zs_strides,
            f"{prefix}_K": np.int64(p.K), f"{prefix}_N": np.int64(p.N)}


def make_proj(rng, ref: Ref, nbits, K, N, g, scale=0.02):
    """RTN-quantised random weights; packing done by the REFERENCE pack kernel and
    checked against the restatement."""
    codes, scs, zes = [], [], []
    for b in nbits:
        W = (rng.standard_normal((N, K)) * scale).astype(np.float16)
        Q, s, z = O.rtn_quantize(W, int(b), g)
        codes.append(Q)
        scs.append(s)
        zes.append(z)
    proj = O.stack_projection(codes, scs, zes, nbits, g, K, N)
    ref_wq = torch.cat([ref.pack(torch.from_numpy(c), int(b)) for c, b in zip(codes, nbits)]).numpy()
    assert np.array_equal(ref_wq, proj.wq), "restated pack disagrees with the reference pack kernel"
    return proj


# --------------------------------------------------------------------------- cases
def case_pack(ref: Ref, out_dir: Path):
    rng = np.random.default_rng(101)
    data = {}
    for nb in (1, 2, 3, 4):
        for (N, K) in ((8, 64), (6, 70), (4, 131), (16, 320)):
            codes = rng.integers(0, 2 ** nb, size=(N, K), dtype=np.uint8)
            packed = ref.pack(torch.from_numpy(codes), nb).numpy()
            # the reference unpack writes whole `unroll` blocks without a mask
            # (utils.py:134,171-172); only call it where that stays in bounds
            unroll = ref.U.highest_divisor(packed.shape[0], max_val=256)
            unpacked = ref.unpack(torch.from_numpy(packed.T.copy()), nb, K).numpy() if K % unroll == 0 else None
            key = f"b{nb}_{N}x{K}"
            data[f"{key}_codes"] = codes
            data[f"{key}_packed"] = packed
            if unpacked is not None:
                data[f"{key}_unpacked"] = unpacked
    np.savez_compressed(out_dir / "pack.npz", **data)
    print("pack.npz", len(data))


def case_group_gemm(ref: Ref, out_dir: Path):
    rng = np.random.default_rng(202)
    data = {}
    for g in (64, 128):
        K, N, M = 256, 128, 5
        bits = [1, 2, 3, 4, 3, 2]
        proj = make_proj(rng, ref, bits, K, N, g)
        x = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
        eye = np.eye(K, dtype=np.float16)
        data.update({f"g{g}_" + k: v for k, v in proj_arrays("w", proj).items()})
        data[f"g{g}_x"] = x
        for mode in ("interp", "gpu"):
            with fma_mode(mode):
                wq, sc, ze, nb, gs, ws, zs = proj_tensors(proj)
                idx_all = torch.arange(len(bits), dtype=torch.int32)
                data[f"g{g}_y_{mode}"] = ref.group_gemm(t(x), idx_all, wq, sc, ze, nb, gs, ws, zs).numpy()
                data[f"g{g}_deq_{mode}"] = ref.group_gemm(t(eye), idx_all, wq, sc, ze, nb, gs, ws, zs).numpy()
    np.savez_compressed(out_dir / "group_gemm.npz", **data)
    print("group_gemm.npz", len(data))


def case_decode_kernels(ref: Ref, out_dir: Path):
    rng = np.random.default_rng(303)
    data = {}
    D, F, g = 256, 128, 64
    bits = [2, 3, 4, 1, 3, 2]
    w1 = make_proj(rng, ref, bits, D, F, g)
    w3 = make_proj(rng, ref, bits, D, F, g)
    w2 = make_proj(rng, ref, bits, F, D, g)
    x = (rng.standard_normal((1, D)) * 0.5).astype(np.float16)
    idx = np.array([4, 0, 2], dtype=np.int32)
    for name, p in (("w1", w1), ("w3", w3), ("w2", w2)):
        data.update(proj_arrays(name, p))
    data["x"], data["idx"] = x, idx
    sh = make_proj(rng, ref, [4], D, 2 * F, g)
    sh2 = make_proj(rng, ref, [3], 2 * F, D, g)
    data.update(proj_arrays("sh", sh))
    data.update(proj_arrays("sh2", sh2))
    xs = (rng.standard_normal((7, D)) * 0.5).astype(np.float16)
    data["xs"] = xs
    h2 = (rng.standard_normal((1, 2 * F)) * 0.1).astype(np.float16)
    data["h2"] = h2
    for mode in ("interp", "gpu"):
        with fma_mode(mode):
            W1, W3, W2 = proj_tensors(w1), proj_tensors(w3), proj_tensors(w2)
            x1, x3 = ref.up_proj(t(x), t(idx), W1[0], W3[0], W1[1], W1[2], W3[1], W3[2], W1[3], W1[5], g)
            x2 = ref.down_proj(x1, x3, t(idx), W2[0], W2[1], W2[2], W2[3], W2[5], g)
            data[f"x1_{mode}"], data[f"x3_{mode}"], data[f"x2_{mode}"] = x1.numpy(), x3.numpy(), x2.numpy()
            S = proj_tensors(sh)
            data[f"gemm_{mode}"] = ref.gemm(t(xs), S[0], S[1], S[2], 4, g).numpy()
            data[f"gemv_{mode}"] = ref.splitk_gemv(t(x), S[0], S[1], S[2], 4, g).numpy()
            S2 = proj_tensors(sh2)
            data[f"gemv2_{mode}"] = ref.splitk_gemv(t(h2), S2[0], S2[1], S2[2], 3, g).numpy()
    np.savez_compressed(out_dir / "decode_kernels.npz", **data)
    print("decode_kernels.npz", len(data))


# --------------------------------------------------------------------------- MoE blocks
def import_moe_block(ref: Ref):
    gl = types.ModuleType("gemlite")
    glc = types.ModuleType("gemlite.core")

    class GemLiteLinearTriton:  # only an isinstance check in from_hf, unused here
        pass

    glc.GemLiteLinearTriton = GemLiteLinearTriton
    gl.core = glc
    sys.modules.setdefault("gemlite", gl)
    sys.modules.setdefault("gemlite.core", glc)
    import transformers.models.deepseek_v2.modeling_deepseek_v2 as ds
    if not hasattr(ds, "DeepseekV2MoE"):
        ds.DeepseekV2MoE = type("DeepseekV2MoE", (torch.nn.Module,), {})
    from gemq.inference import moe_block as mb

    def dgg(x, indices, wq, scales, zeros, nbits, group_sizes, wq_strides, zs_strides, compute_dtype=torch.float16):
        return ref.group_gemm(x.contiguous(), indices.reshape(-1).to(torch.int32), wq, scales, zeros, nbits,
                              group_sizes, wq_strides, zs_strides)

    def dg(x, w_q, scales, zeros, nbits, group_size):
        return ref.gemm(x.contiguous(), w_q, scales, zeros, nbits, group_size)

    def gv(x, w_q, scales, zeros, nbits, group_size):
        return ref.splitk_gemv(x.contiguous(), w_q, scales, zeros, nbits, group_size)

    def up(x, idx, w1, w3, w1_scales, w1_zeros, w3_scales, w3_zeros, nbits, w_strides, group_size):
        return ref.up_proj(x.contiguous(), idx.to(torch.int32), w1, w3, w1_scales, w1_zeros, w3_scales, w3_zeros,
                           nbits, w_strides, group_size)

    def down(x1, x3, idx, w2, w2_scales, w2_zeros, nbits, w_strides, group_size):
        return ref.down_proj(x1, x3, idx.to(torch.int32), w2, w2_scales, w2_zeros, nbits, w_strides, group_size)

    mb.dequant_group_gemm_triton = dgg
    mb.dequant_gemm_triton = dg
    mb.dequant_splitk_gemv_triton = gv
    mb.fused_dequant_up_proj_triton = up
    mb.fused_dequant_down_proj_triton = down
    return mb


FAMILIES = {
    # name: (class, norm_topk_prob, shared)
    "olmoe": ("QuantFusedOlmoeMoEBlock", False, False),
    "qwen3": ("QuantFusedQwen3MoeMoEBlock", True, False),
    "mixtral": ("QuantFusedMixtralMoEBlock", True, False),
    "deepseek": ("QuantFusedDeepseekV2MoEBlock", False, True),
}

# same per-expert bit pattern as the reference's block test (test_moe_block_equiv.py:37)
BLOCK_BITS = [1, 2, 3, 2, 3, 1, 2, 3]


def build_block(mb, family: str, blk: O.BlockWeights, D: int, F: int, g: int):
    cls_name, norm, shared = FAMILIES[family]
    cls = getattr(mb, cls_name)
    b = cls.__new__(cls)
    torch.nn.Module.__init__(b)
    b.hidden_dim, b.ffn_dim = D, F
    b.num_experts, b.top_k = blk.w1.num_experts, blk.top_k
    b.norm_topk_prob = norm
    b.gate = torch.nn.Linear(D, b.num_experts, bias=False).half()
    b.gate.weight.data = t(blk.gate_w)
    for name in ("w1", "w2", "w3"):
        p = getattr(blk, name)
        for attr, val in zip(("wq", "scales", "zeros", "nbits", "group_sizes", "wq_strides", "zs_strides"),
                             proj_tensors(p)):
            setattr(b, f"{name}_{attr}", val)
    b.block_group_size = g
    if shared:
        b.num_shared_experts = 2
        for name, p in (("shared_w1", blk.shared_w1), ("shared_w3", blk.shared_w3), ("shared_w2", blk.shared_w2)):
            wq, sc, ze, *_ = proj_tensors(p)
            setattr(b, f"{name}_wq", wq)
            setattr(b, f"{name}_scales", sc)
            setattr(b, f"{name}_zeros", ze)
        b.shared_nbits = int(blk.shared_w1.nbits[0])
        b.shared_group_size = g
    return b


def case_blocks(ref: Ref, out_dir: Path):
    mb = import_moe_block(ref)
    D, F, E, k, g, T = 256, 256, 8, 2, 64, 12
    for fi, family in enumerate(FAMILIES):
        rng = np.random.default_rng(400 + fi)
        _, norm, shared = FAMILIES[family]
        w1 = make_proj(rng, ref, BLOCK_BITS, D, F, g)
        w3 = make_proj(rng, ref, BLOCK_BITS, D, F, g)
        w2 = make_proj(rng, ref, BLOCK_BITS, F, D, g)
        gate = (rng.standard_normal((E, D)) * 0.02).astype(np.float16)
        blk = O.BlockWeights(gate_w=gate, w1=w1, w3=w3, w2=w2, top_k=k, norm_topk_prob=norm,
                             router_fp32=(family == "deepseek"))
        data = {"gate_w": gate, "D": np.int64(D), "F": np.int64(F), "top_k": np.int64(k),
                "group_size": np.int64(g), "norm_topk_prob": np.int64(norm)}
        if shared:
            blk.shared_w1 = make_proj(rng, ref, [3], D, 2 * F, g)
            blk.shared_w3 = make_proj(rng, ref, [3], D, 2 * F, g)
            blk.shared_w2 = make_proj(rng, ref, [3], 2 * F, D, g)
            for name in ("shared_w1", "shared_w3", "shared_w2"):
                data.update(proj_arrays(name, getattr(blk, name)))
        for name in ("w1", "w3", "w2"):
            data.update(proj_arrays(name, getattr(blk, name)))
        x = (rng.standard_normal((1, T, D)) * 0.5).astype(np.float16)
        x1 = (rng.standard_normal((1, 1, D)) * 0.5).astype(np.float16)
        data["x"], data["x_one"] = x[0], x1[0]
        b = build_block(mb, family, blk, D, F, g)
        # routing decisions, recomputed with the same torch ops the block runs
        # (moe_block.py:790-797, 549-556; one-token 828-833, 280-283, 591-597)
        with torch.no_grad():
            xt = t(x[0])
            if family == "deepseek":
                lg = torch.nn.functional.linear(xt.float(), b.gate.weight.float())
            else:
                lg = b.gate(xt)
            rw = torch.softmax(lg, dim=1, dtype=torch.float)
            rw, sel = torch.topk(rw, k, dim=-1)
            if norm:
                rw /= rw.sum(dim=-1, keepdim=True)
            data["route_logits"] = lg.float().numpy()
            data["route_idx"], data["route_w"] = sel.numpy(), rw.to(torch.float16).numpy()
            x1t = t(x1[0])
            if family == "deepseek":
                lg1 = torch.nn.functional.linear(x1t.float(), b.gate.weight.float())
                p1 = torch.softmax(lg1, dim=1, dtype=torch.float)
            elif family == "mixtral":
                lg1 = b.gate(x1t)
                p1 = torch.softmax(lg1, dim=-1)
            else:
                lg1 = b.gate(x1t)
                p1 = torch.softmax(lg1, dim=1, dtype=torch.float)
            p1, sel1 = torch.topk(p1, k, dim=-1)
            if norm:
                p1 /= p1.sum(dim=-1, keepdim=True)
            data["route1_idx"], data["route1_w"] = sel1.numpy(), p1.to(torch.float16).numpy()
        for mode in ("interp", "gpu"):
            with fma_mode(mode), torch.no_grad():
                yn = b.forward_n_tokens(t(x))
                yn = yn[0] if isinstance(yn, tuple) else yn
                y1 = b.forward_one_token(t(x1))
                y1 = y1[0] if isinstance(y1, tuple) else y1
                data[f"y_ntok_{mode}"] = yn.reshape(T, D).numpy()
                data[f"y_one_{mode}"] = y1.reshape(1, D).numpy()
        np.savez_compressed(out_dir / f"block_{family}.npz", **data)
        print(f"block_{family}.npz", len(data))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to a RobustGEMQ checkout")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    torch.manual_seed(0)
    ref = Ref(args.reference)
    out_dir = Path(args.out)
    case_pack(ref, out_dir)
    case_group_gemm(ref, out_dir)
    case_decode_kernels(ref, out_dir)
    case_blocks(ref, out_dir)


if __name__ == "__main__":
    main()
