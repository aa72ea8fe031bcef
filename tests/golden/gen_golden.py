"""Generate golden fixtures from the reference's own Python code.

Run in a container that has the reference checkout (its path given by
``--reference`` or the VC_REFERENCE_ROOT environment variable).  It imports, by path:
  * third_party/sageattention_local/sageattention_local/vc_reference.py
    (the reference's decoded-payload FP32 oracle),
  * third_party/sageattention_local/sageattention_local/triton/quant_per_thread.py
    (the reference's Triton INT8 quantiser, executed on CPU with
    TRITON_INTERPRET=1),
  * src/vc_attention/core.py (the reference backend of the Config API),
and writes small ``.npz`` fixtures next to this script.  The fixtures are
committed; nothing on a GPU box reads the reference.

Usage:  python tests/golden/gen_golden.py --reference <path-to-reference>
"""
import argparse
import importlib.util
import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
from oracle import vc_oracle as O  # noqa: E402
sys.path.insert(0, str(HERE))
from inputs import qk_inputs, mixture_values  # noqa: E402


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sage_state(st):
    """Oracle state -> the reference's layout/types for vc_reference.reference."""
    v8 = O.to_sage_layout(st["v"])
    return {**st, "v": torch.from_numpy(v8).view(torch.float8_e4m3fn),
            "means": torch.from_numpy(np.asarray(st["means"])) if np.size(st["means"]) else torch.empty(0, dtype=torch.float16)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VC_REFERENCE_ROOT"),
                    help="path of the reference checkout (or set VC_REFERENCE_ROOT)")
    ap.add_argument("--hadamard", action="store_true",
                    help="only (re)write the Hadamard / E4M3 block-QK fixtures (step 5)")
    ap.add_argument("--config-defaults", action="store_true",
                    help="only (re)write the Config-default fixtures (step 6)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path-to-reference> or set VC_REFERENCE_ROOT")
    ref = Path(args.reference)
    if args.hadamard or args.config_defaults:
        sys.path.insert(0, str(ref / "src"))
        from vc_attention import core
        manifest = json.loads((HERE / "manifest.json").read_text())
        if args.hadamard:
            hadamard_fixtures(core, manifest)
        if args.config_defaults:
            config_default_fixtures(core, manifest)
        (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, default=str) + "\n")
        return
    sage = ref / "third_party/sageattention_local/sageattention_local"
    vc_ref = load(sage / "vc_reference.py", "ref_vc_reference")
    qpt = load(sage / "triton/quant_per_thread.py", "ref_quant_per_thread")
    sys.path.insert(0, str(ref / "src"))
    from vc_attention import core  # the reference package, loaded from the checkout

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    manifest = {}

    # 1. ExpCast codes on a dense sweep plus specials (both reference functions).
    shifted = torch.cat((torch.linspace(-15, 1, 65537), torch.tensor([-float("inf"), -20., 0., 1., -1e30])))
    codes_sage = vc_ref.expcast_codes(shifted).numpy()
    codes_core = core.expcast_codes(shifted).numpy()
    np.savez_compressed(HERE / "expcast.npz", shifted=shifted.numpy(), codes=codes_sage, codes_core=codes_core)
    manifest["expcast"] = {"n": int(shifted.numel()), "core_equals_sage": bool((codes_sage == codes_core).all())}

    # 2. INT8 Q/K payloads from the reference Triton kernels (interpreted on CPU).
    qk_cases = {
        "c1_fp32": (0, (1, 2, 1024, 128), torch.float32, 2 ** 0.5, 0.0),
        "tail_bf16_d64": (1, (1, 2, 200, 64), torch.bfloat16, 3 ** 0.5, 0.0),
        "tail_fp16_d128": (2, (2, 1, 129, 128), torch.float16, 1.0, 0.0),
        "single_bf16": (3, (1, 1, 1, 64), torch.bfloat16, 0.0, 0.0),
        "outlier_bf16": (4, (1, 3, 257, 128), torch.bfloat16, 3 ** 0.5, 0.01),
    }
    for name, (seed, shape, dtype, koff, outl) in qk_cases.items():
        q, k, v = qk_inputs(seed, shape, dtype, koff, outl)
        km = k.mean(dim=2, keepdim=True)
        q8, qs, k8, ks = qpt.per_thread_int8(q, k, km, BLKQ=64, WARPQ=16, BLKK=128, WARPK=128, tensor_layout="HND")
        np.savez_compressed(HERE / f"qk_{name}.npz", seed=seed, shape=shape, koff=koff, outliers=outl,
                            dtype=str(dtype).split(".")[-1], km=km.float().numpy(), q8=q8.numpy(),
                            qs=qs.numpy(), k8=k8.numpy(), ks=ks.numpy())
        manifest[f"qk_{name}"] = {"shape": list(shape), "dtype": str(dtype)}

    # 3. Attention outputs of the reference oracle on oracle-prepared payloads.
    att_cases = {
        # name: seed, shape, dtype, koff, expcast, v_smooth, v_scale_mode, queries
        "c1_expcast": (0, (1, 2, 1024, 128), torch.float32, 2 ** 0.5, True, False, "channel", None),
        "tail_expcast_d64": (5, (1, 2, 300, 64), torch.bfloat16, 3 ** 0.5, True, False, "channel", None),
        "smooth_channel": (6, (1, 2, 300, 128), torch.bfloat16, 3 ** 0.5, True, True, "channel", None),
        "smooth_block_d64": (7, (2, 1, 257, 64), torch.float16, 1.0, True, True, "block", None),
        "control_no_expcast": (8, (1, 1, 129, 128), torch.bfloat16, 1.0, False, False, "channel", None),
    }
    for name, (seed, shape, dtype, koff, cast, smooth, vmode, qi) in att_cases.items():
        q, k, v = qk_inputs(seed, shape, dtype, koff)
        if smooth:
            v = mixture_values(seed, shape, dtype)
        st = O.prepare(q, k, v, expcast=cast, v_smooth=smooth, v_scale_mode=vmode)
        out = vc_ref.reference(sage_state(st), query_indices=qi)
        dense = O.dense_attention(q, k, v)
        np.savez_compressed(HERE / f"att_{name}.npz", seed=seed, shape=shape, koff=koff,
                            dtype=str(dtype).split(".")[-1], expcast=cast, v_smooth=smooth, v_scale_mode=vmode,
                            permutation=(st["permutation"].numpy() if st["permutation"] is not None else np.zeros(0, np.int64)),
                            out=out.numpy())
        manifest[f"att_{name}"] = {"shape": list(shape), "dtype": str(dtype), "expcast": cast, "v_smooth": smooth,
                                   "vs_dense": O.metrics(out, dense)}

    # 4. Boundary A: the Config API reference backend (INT8 path differs in QK
    #    format, so these are tolerance fixtures).
    cfg_cases = {
        "c1_cfg_expcast": (0, (1, 2, 1024, 128), torch.float32, 2 ** 0.5, dict(expcast=True, qk_hadamard=False)),
        "cfg_smooth": (9, (1, 2, 384, 64), torch.float32, 1.0, dict(expcast=True, v_smooth=True, qk_hadamard=False)),
    }
    for name, (seed, shape, dtype, koff, kw) in cfg_cases.items():
        q, k, v = qk_inputs(seed, shape, dtype, koff)
        out, counters = core.attention(q, k, v, core.Config(backend="reference", **kw))
        np.savez_compressed(HERE / f"{name}.npz", seed=seed, shape=shape, koff=koff, out=out.numpy(),
                            config=json.dumps(kw))
        manifest[name] = {"shape": list(shape), "config": kw, "counters": {k2: v2 for k2, v2 in counters.items()}}

    hadamard_fixtures(core, manifest)
    config_default_fixtures(core, manifest)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, default=str) + "\n")
    print(json.dumps(manifest, indent=1, default=str))


def hadamard_fixtures(core, manifest):
    """5. The Config contract's own QK path (qk_hadamard=True): Q/K payloads
    from the reference's preprocess_qk + _encode per block, and reference
    backend outputs of core.attention."""
    cases = {"hadamard_qk": (21, (1, 2, 300, 128), torch.bfloat16, 2 ** 0.5, 256),
             "hadamard_qk_d64": (22, (2, 1, 517, 64), torch.float16, 1.0, 128)}
    for name, (seed, shape, dtype, koff, kqb) in cases.items():
        q, k, _ = qk_inputs(seed, shape, dtype, koff)
        km = k.float().mean(dim=-2)
        qh, kh = core.preprocess_qk(q, k, k_smooth=True, qk_hadamard=True)
        out = {}
        for tag, x, block in (("q", qh, 128), ("k", kh, kqb)):
            bits, scales = [], []
            for start in range(0, x.shape[-2], block):
                payload, scale = core._encode(x[..., start:start + block, :], (-2, -1))
                bits.append(payload.view(torch.uint8))
                scales.append(scale.reshape(*x.shape[:-2], 1))
            out[tag + "8"] = torch.cat(bits, dim=-2).numpy()
            out[tag + "s"] = torch.cat(scales, dim=-1).numpy()
        np.savez_compressed(HERE / f"{name}.npz", seed=seed, shape=shape, koff=koff, dtype=str(dtype).split(".")[-1],
                            k_quant_block=kqb, km=km.numpy(), **out)
        manifest[name] = {"shape": list(shape), "dtype": str(dtype), "k_quant_block": kqb}
    cfg_cases = {
        "cfg_hadamard": (23, (1, 2, 640, 128), torch.float32, 2 ** 0.5, dict(expcast=True, qk_hadamard=True)),
        "cfg_hadamard_smooth": (24, (1, 2, 500, 64), torch.float32, 1.0,
                                dict(expcast=True, v_smooth=True, qk_hadamard=True, k_quant_block=128)),
    }
    for name, (seed, shape, dtype, koff, kw) in cfg_cases.items():
        q, k, v = qk_inputs(seed, shape, dtype, koff)
        out, counters = core.attention(q, k, v, core.Config(backend="reference", **kw))
        np.savez_compressed(HERE / f"{name}.npz", seed=seed, shape=shape, koff=koff, out=out.numpy(),
                            config=json.dumps(kw))
        manifest[name] = {"shape": list(shape), "config": kw, "counters": {k2: v2 for k2, v2 in counters.items()}}


def config_default_fixtures(core, manifest):
    """6. The Config contract with the reference's defaults (no ExpCast: the
    FP8-P control with exact exp row sums; Hadamard E4M3 block Q/K; V
    encoded per 128-token tile) and its INT8-QK control: reference backend
    outputs of core.attention."""
    cases = {
        "cfg_default": (25, (1, 2, 640, 128), torch.float32, 2 ** 0.5, {}),
        "cfg_default_smooth": (26, (1, 2, 500, 64), torch.float32, 1.0, dict(v_smooth=True)),
        "cfg_control_int8": (27, (1, 2, 384, 128), torch.float32, 2 ** 0.5, dict(qk_hadamard=False)),
    }
    for name, (seed, shape, dtype, koff, kw) in cases.items():
        q, k, v = qk_inputs(seed, shape, dtype, koff)
        out, counters = core.attention(q, k, v, core.Config(backend="reference", **kw))
        np.savez_compressed(HERE / f"{name}.npz", seed=seed, shape=shape, koff=koff, out=out.numpy(),
                            config=json.dumps(kw))
        manifest[name] = {"shape": list(shape), "config": kw, "counters": {k2: v2 for k2, v2 in counters.items()}}


if __name__ == "__main__":
    main()
