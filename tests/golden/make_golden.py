"""Generate golden fixtures by running the REFERENCE implementation on CPU.

Run in a container that has the reference checkout (read-only is fine):

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py --reference /path/to/metal_liger

The reference is imported as the package ``metal_liger`` through a symlink in
a temporary directory (its modules use absolute ``metal_liger.*`` imports).
Every case draws seeded inputs, runs the reference's own autograd Function
forward and backward (the same calls its tests/test_fused_ops.py makes), and
stores inputs + outputs in ``tests/golden/<case>.pt``.  The fixtures are small
(a few KB to a few hundred KB) so they can be committed; the GPU box never
needs the reference.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def import_reference(ref_dir: Path):
    tmp = Path(tempfile.mkdtemp(prefix="mlref_"))
    (tmp / "metal_liger").symlink_to(ref_dir)
    sys.path.insert(0, str(tmp))
    import metal_liger  # noqa: F401
    from metal_liger.ops import fused_rms_norm, fused_swiglu, fused_rope
    from metal_liger.ops import fused_linear_cross_entropy, fused_lora
    return fused_rms_norm, fused_swiglu, fused_rope, fused_linear_cross_entropy, fused_lora


def leaf(t):
    return t.detach().clone().requires_grad_(True)


def case_rms(mod, seed, shape, x_dtype, w_dtype, eps=1e-6):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g).to(x_dtype)
    w = (1.0 + 0.1 * torch.randn(shape[-1], generator=g)).to(w_dtype)
    dy = torch.randn(*shape, generator=g).to(x_dtype)
    xl, wl = leaf(x), leaf(w)
    y = mod._FusedRMSNormFunction.apply(xl, wl, eps)
    y.backward(dy)
    return dict(x=x, w=w, dy=dy, eps=torch.tensor(eps), y=y.detach(), dx=xl.grad, dw=wl.grad)


def case_swiglu(mod, seed, shape, dtype):
    g = torch.Generator().manual_seed(seed)
    gate = torch.randn(*shape, generator=g).to(dtype)
    up = torch.randn(*shape, generator=g).to(dtype)
    dy = torch.randn(*shape, generator=g).to(dtype)
    gl, ul = leaf(gate), leaf(up)
    out = mod._FusedSwiGLUFunction.apply(gl, ul)
    out.backward(dy)
    return dict(gate=gate, up=up, dy=dy, out=out.detach(), dgate=gl.grad, dup=ul.grad)


def cos_sin_ref_test(seq, dim, theta):
    # The reference test's table construction (tests/test_fused_ops.py:146-154).
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))
    ang = torch.arange(seq).float()[:, None] * freqs[None, :]
    return torch.cos(ang).repeat(1, 2), torch.sin(ang).repeat(1, 2)


def case_rope(mod, seed, shape, dtype, theta, table="ref"):
    g = torch.Generator().manual_seed(seed)
    b, h, s, d = shape
    x = torch.randn(*shape, generator=g).to(dtype)
    dy = torch.randn(*shape, generator=g)
    if table == "ref":
        cos, sin = cos_sin_ref_test(s, d, theta)
    else:  # HF-style [B, 1, S, D] tables from per-batch positions, cast to x dtype
        pos = torch.stack([torch.arange(s) + 3 * i for i in range(b)])
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
        fr = pos.float()[..., None] * inv
        emb = torch.cat((fr, fr), -1)
        cos, sin = emb.cos()[:, None].to(dtype), emb.sin()[:, None].to(dtype)
    out_dtype = torch.promote_types(dtype, cos.dtype)
    dy = dy.to(out_dtype)
    xl = leaf(x)
    y = mod._FusedRoPEFunction.apply(xl, cos, sin)
    y.backward(dy)
    return dict(x=x, cos=cos, sin=sin, dy=dy, y=y.detach(), dx=xl.grad)


def case_flce(mod, seed, n, h, v, chunk, ignore_frac, with_bias=False, all_ignored=False):
    g = torch.Generator().manual_seed(seed)
    hid = torch.randn(n, h, generator=g)
    w = 0.02 * torch.randn(v, h, generator=g) * 10
    labels = torch.randint(0, v, (n,), generator=g)
    nign = int(round(ignore_frac * n))
    if all_ignored:
        labels[:] = -100
    elif nign:
        idx = torch.randperm(n, generator=g)[:nign]
        labels[idx] = -100
    bias = 0.1 * torch.randn(v, generator=g) if with_bias else None
    hl, wl = leaf(hid), leaf(w)
    loss = mod._FusedLinearCrossEntropyFunction.apply(hl, wl, labels, bias, -100, chunk)
    go = torch.tensor(1.7)
    loss.backward(go)
    out = dict(hidden=hid, weight=w, labels=labels, chunk=torch.tensor(chunk),
               grad_output=go, loss=loss.detach(), dhidden=hl.grad, dweight=wl.grad)
    if bias is not None:
        out["bias"] = bias
    return out


def lora_params(g, out_f, in_f, r, s, dtype):
    w = (0.02 * torch.randn(out_f, in_f, generator=g) * 5).to(dtype)
    a = (0.1 * torch.randn(r, in_f, generator=g)).to(dtype)
    b = (0.1 * torch.randn(out_f, r, generator=g)).to(dtype)
    return w, a, b, s


def case_lora_qkv(mod, seed, x_shape, q_out, kv_out, r, s, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*x_shape, generator=g).to(dtype)
    hdim = x_shape[-1]
    q = lora_params(g, q_out, hdim, r, s, dtype)
    k = lora_params(g, kv_out, hdim, r, s, dtype)
    v = lora_params(g, kv_out, hdim, r, s, dtype)
    dq = torch.randn(*x_shape[:-1], q_out, generator=g).to(dtype)
    dk = torch.randn(*x_shape[:-1], kv_out, generator=g).to(dtype)
    dv = torch.randn(*x_shape[:-1], kv_out, generator=g).to(dtype)
    xl = leaf(x)
    ql = [leaf(t) if torch.is_tensor(t) else t for t in q]
    kl = [leaf(t) if torch.is_tensor(t) else t for t in k]
    vl = [leaf(t) if torch.is_tensor(t) else t for t in v]
    Q, K, V = mod._LoRA_QKV.apply(xl, *ql, *kl, *vl)
    torch.autograd.backward([Q, K, V], [dq, dk, dv])
    out = dict(x=x, dq=dq, dk=dk, dv=dv, s=torch.tensor(s), Q=Q.detach(), K=K.detach(),
               V=V.detach(), dx=xl.grad)
    for name, p in (("q", ql), ("k", kl), ("v", vl)):
        out[f"{name}_w"], out[f"{name}_a"], out[f"{name}_b"] = p[0].detach(), p[1].detach(), \
            p[2].detach()
        out[f"{name}_da"], out[f"{name}_db"] = p[1].grad, p[2].grad
    return out


def case_lora_mlp(mod, seed, x_shape, inter, r, s, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*x_shape, generator=g).to(dtype)
    hdim = x_shape[-1]
    gp = lora_params(g, inter, hdim, r, s, dtype)
    up = lora_params(g, inter, hdim, r, s, dtype)
    dp = lora_params(g, hdim, inter, r, s, dtype)
    dy = torch.randn(*x_shape, generator=g).to(dtype)
    xl = leaf(x)
    gl = [leaf(t) if torch.is_tensor(t) else t for t in gp]
    ul = [leaf(t) if torch.is_tensor(t) else t for t in up]
    dl = [leaf(t) if torch.is_tensor(t) else t for t in dp]
    out_t = mod._LoRA_MLP.apply(xl, *gl, *ul, *dl)
    out_t.backward(dy)
    out = dict(x=x, dy=dy, s=torch.tensor(s), out=out_t.detach(), dx=xl.grad)
    for name, p in (("gate", gl), ("up", ul), ("down", dl)):
        out[f"{name}_w"], out[f"{name}_a"], out[f"{name}_b"] = p[0].detach(), p[1].detach(), \
            p[2].detach()
        out[f"{name}_da"], out[f"{name}_db"] = p[1].grad, p[2].grad
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("METAL_LIGER_REF"),
                    help="directory of the reference package (or METAL_LIGER_REF)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference (or METAL_LIGER_REF): the reference package's directory")
    rms, swi, rope, flce, lora = import_reference(Path(args.reference))
    torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))
    cases = {
        "rms_f32": lambda: case_rms(rms, 101, (2, 16, 256), torch.float32, torch.float32),
        "rms_f32_odd": lambda: case_rms(rms, 102, (3, 5, 300), torch.float32, torch.float32),
        "rms_f32_row1": lambda: case_rms(rms, 103, (1, 1024), torch.float32, torch.float32),
        "rms_bf16_wf32": lambda: case_rms(rms, 104, (4, 8, 512), torch.bfloat16, torch.float32),
        "rms_bf16": lambda: case_rms(rms, 105, (4, 8, 512), torch.bfloat16, torch.bfloat16),
        "swiglu_f32": lambda: case_swiglu(swi, 201, (2, 16, 512), torch.float32),
        "swiglu_bf16_odd": lambda: case_swiglu(swi, 202, (3, 7, 99), torch.bfloat16),
        "swiglu_bf16": lambda: case_swiglu(swi, 203, (2, 8, 768), torch.bfloat16),
        "rope_f32_reftable": lambda: case_rope(rope, 301, (2, 8, 32, 64), torch.float32, 10000.0),
        "rope_bf16_hf": lambda: case_rope(rope, 302, (2, 4, 16, 128), torch.bfloat16, 5e6,
                                          table="hf"),
        "rope_bf16_promote": lambda: case_rope(rope, 303, (1, 2, 8, 32), torch.bfloat16,
                                               10000.0),
        "flce_f32": lambda: case_flce(flce, 401, 64, 32, 1000, 256, 0.1),
        "flce_f32_bias": lambda: case_flce(flce, 402, 48, 24, 777, 128, 0.25, with_bias=True),
        "flce_f32_allign": lambda: case_flce(flce, 403, 16, 32, 300, 128, 0.0,
                                             all_ignored=True),
        "lora_qkv_f32": lambda: case_lora_qkv(lora, 42, (2, 16, 128), 128, 128, 8, 2.0,
                                              torch.float32),
        "lora_qkv_gqa_f32": lambda: case_lora_qkv(lora, 501, (2, 8, 64), 64, 16, 4, 2.0,
                                                  torch.float32),
        "lora_mlp_f32": lambda: case_lora_mlp(lora, 601, (2, 8, 64), 96, 4, 2.0, torch.float32),
    }
    out = Path(args.out)
    for name, fn in cases.items():
        data = fn()
        data = {k: v.detach().contiguous() for k, v in data.items()}
        torch.save(data, out / f"{name}.pt")
        size = sum(v.numel() * v.element_size() for v in data.values())
        print(f"{name}: {len(data)} tensors, {size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
