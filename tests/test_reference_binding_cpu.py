"""The B200 path bound into the reference runtime itself, on CPU.

Every check runs in a fresh interpreter whose path holds the reference's own
package (installed into baseline/_ref by ``oracle/build_ref.py``, or the
reference source tree), so the reference's registries, protocols, value types,
diffusers bridge and Wan installer are the real ones; a fake ``diffusers``
module stands in for the library the way the reference's own tests fake it
(reference tests/test_wan.py:31-93).  A compute-capability 10.0 device is
simulated by forcing availability, since there is no GPU here.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

from oracle.build_ref import installed_reference_path, reference_root  # noqa: E402


def _reference_path() -> list[str] | None:
    p = installed_reference_path()
    if p is not None:
        return [str(p)]
    root = reference_root()
    if root is not None:
        return [str(root / "src"), str(root / "kernels")]
    return None


REF_PATH = _reference_path()
pytestmark = pytest.mark.skipif(REF_PATH is None, reason="reference package not installed")

# A fake diffusers: the attention-dispatch registry the reference's bridge
# writes into (diffusers_backend.py:289-361) and the Wan processor import
# path its installer resolves (wan_processor.py:98-108).
FAKE_DIFFUSERS = textwrap.dedent(
    """
    import enum, sys, types

    def _mod(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__["__path__"] = []
        m.__dict__.update(attrs)
        sys.modules[name] = m
        return m

    class AttentionBackendName(str, enum.Enum):
        NATIVE = "native"

    class _AttentionBackendRegistry:
        _backends = {AttentionBackendName.NATIVE: lambda *a, **k: "native"}
        _constraints = {}
        _supported_arg_names = {}
        _active_backend = AttentionBackendName.NATIVE

        @classmethod
        def set_active_backend(cls, backend):
            cls._active_backend = backend

    def dispatch_attention_fn(query, key, value, backend=None, **kw):
        name = backend if backend is not None else _AttentionBackendRegistry._active_backend
        return _AttentionBackendRegistry._backends[name](query, key, value, **kw)

    class WanAttnProcessor:
        _attention_backend = None

    _mod("diffusers")
    _mod("diffusers.models")
    _mod("diffusers.models.attention_dispatch", AttentionBackendName=AttentionBackendName,
         _AttentionBackendRegistry=_AttentionBackendRegistry,
         dispatch_attention_fn=dispatch_attention_fn)
    _mod("diffusers.models.transformers")
    _mod("diffusers.models.transformers.transformer_wan", WanAttnProcessor=WanAttnProcessor)
    """
)

# Forces "a B200 is present" for the B200 op and backend on this CPU host.
FORCE_B200 = textwrap.dedent(
    """
    import repercep_runtime_b200.attention.fp8_b200 as _f
    from repercep_runtime_b200.backend.b200 import B200Backend
    from repercep_runtime_b200.hardware import B200, DeviceSpec
    _f.b200_device_present = lambda: True
    B200Backend.is_available = lambda self: True
    B200Backend.devices = lambda self: (DeviceSpec(0, B200, "NVIDIA B200", 183 << 30, 148),)
    """
)


def run(*parts: str, env_extra: dict[str, str] | None = None) -> dict:
    """Run the script made of ``parts`` (each dedented on its own) with the
    reference on the path; return the JSON object its last line prints."""
    script = "\n".join(textwrap.dedent(p) for p in parts)
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([*REF_PATH, str(REPO)])
    env.pop("REPERCEP_FP8_ATTENTION", None)
    env.update(env_extra or {})
    proc = subprocess.run([sys.executable, "-c", script], env=env,
                          capture_output=True, text=True, timeout=240, cwd=str(REPO))
    assert proc.returncode == 0, proc.stderr[-3000:]
    return json.loads(proc.stdout.strip().splitlines()[-1])


def test_value_types_are_the_references_own():
    r = run(
        """
        import json
        import repercep.hardware as rh, repercep.attention.types as rt
        import repercep_runtime_b200.hardware as h
        from repercep_runtime_b200.attention import AttentionShape
        from repercep_runtime_b200.backend.b200 import arch_for_capability
        print(json.dumps({
            "dtype": h.DType is rh.DType, "vendor": h.Vendor is rh.Vendor,
            "arch": type(h.B200) is rh.DeviceArch, "shape": AttentionShape is rt.AttentionShape,
            "b200_vendor_is": arch_for_capability(10, 0).vendor is rh.Vendor.NVIDIA,
            "flag": h.REFERENCE_TYPES}))
        """
    )
    assert all(r.values()), r


def test_supports_takes_the_references_shape_and_dtype():
    r = run(
        FORCE_B200,
        """
        import json
        from repercep.attention.types import AttentionKind, AttentionShape
        from repercep.hardware import DType
        from repercep.attention.protocol import AttentionOp
        from repercep_runtime_b200.attention import B200FP8Attention
        op = B200FP8Attention()
        s = lambda *a: op.supports(AttentionShape(*a), DType.BF16)
        print(json.dumps({
            "protocol": isinstance(op, AttentionOp),
            "self": s(2, 32, 57600, 57600, 128),
            "cross_full": s(2, 32, 4096, 1024, 128),
            "cross_causal": s(2, 32, 4096, 1024, 128, AttentionKind.CAUSAL),
            "causal": s(2, 32, 4096, 4096, 128, AttentionKind.CAUSAL),
            "neighborhood": s(2, 32, 4096, 4096, 128, AttentionKind.NEIGHBORHOOD),
            "fp16": op.supports(AttentionShape(1, 8, 4096, 4096, 64), DType.FP16),
            "fp32": op.supports(AttentionShape(1, 8, 4096, 4096, 64), DType.FP32),
            "d96": s(1, 8, 4096, 4096, 96)}))
        """
    )
    assert r == {"protocol": True, "self": True, "cross_full": True, "cross_causal": False,
                 "causal": True, "neighborhood": False, "fp16": True, "fp32": False, "d96": False}


def test_reference_backend_registry_selects_the_b200_backend_and_op():
    r = run(
        FORCE_B200,
        """
        import json
        import repercep.backend.registry as breg
        from repercep.backend.protocol import Backend
        from repercep.attention.types import AttentionShape
        from repercep.hardware import DType
        from repercep_runtime_b200 import integration
        before = breg.select_backend().name if breg.available_backends() else None
        done = integration.install()
        again = integration.install()
        b = breg.select_backend()
        op = b.attention_op(AttentionShape(2, 32, 57600, 57600, 128), DType.BF16)
        odd = b.attention_op(AttentionShape(2, 32, 4096, 4096, 96), DType.BF16)
        print(json.dumps({
            "before": before, "order": [x.name for x in breg._ALL_BACKENDS],
            "backend": b.name, "protocol": isinstance(b, Backend), "op": op.name,
            "odd": odd.name, "fp8_cap": b.capabilities().supports_fp8,
            "pinned": breg.select_backend("cuda-b200").name,
            "idempotent": again["backend"] == "present" and again["attention"] == "present"}))
        """,
        env_extra={"REPERCEP_FP8_ATTENTION": "1"},
    )
    assert r["before"] != "cuda-b200"
    assert r["order"].index("cuda-b200") < r["order"].index("cuda")
    assert r["backend"] == "cuda-b200" and r["protocol"] and r["pinned"] == "cuda-b200"
    assert r["op"] == "fp8-b200-flash"
    assert r["odd"] != "fp8-b200-flash"  # head dim 96 falls through to the reference's chain
    assert r["fp8_cap"] and r["idempotent"]


def test_reference_select_attention_op_routes_b200_archs():
    """The reference's own function (and the CUDA backend module's copy of
    it) picks the B200 op for the arch the reference's CUDABackend reports on
    a B200 (gfx_id "100"), only with FP8 enabled."""
    script = (
        FORCE_B200,
        """
        import json
        import repercep.attention.registry as areg
        import repercep.backend.cuda as cuda
        from repercep.attention.types import AttentionShape
        from repercep.hardware import H100, DeviceArch, DType, Vendor
        from repercep_runtime_b200 import integration
        integration.install()
        shape = AttentionShape(2, 32, 57600, 57600, 128)
        cc100 = DeviceArch(Vendor.NVIDIA, "100", "unknown")
        print(json.dumps({
            "ref_cc100": areg.select_attention_op(cc100, shape, DType.BF16).name,
            "cuda_module": cuda.select_attention_op(cc100, shape, DType.BF16).name,
            "h100": areg.select_attention_op(H100, shape, DType.BF16).name}))
        """
    )
    on = run(*script, env_extra={"REPERCEP_FP8_ATTENTION": "1"})
    assert on["ref_cc100"] == "fp8-b200-flash" and on["cuda_module"] == "fp8-b200-flash"
    assert on["h100"] != "fp8-b200-flash"
    off = run(*script)
    assert "fp8-b200-flash" not in off.values()
    te = run(*script, env_extra={"REPERCEP_FP8_ATTENTION": "te"})
    assert te["ref_cc100"] != "fp8-b200-flash"


@pytest.mark.parametrize("order", ["reference_first", "b200_first"])
def test_diffusers_seam_reaches_the_b200_bridge(order):
    """Whichever registers first, diffusers' "repercep_fp8" entry ends up as
    this package's function, the reference's Wan installer and Cosmos
    activation reach it, and it keeps the reference's function as the
    hand-off for calls the B200 kernel does not serve."""
    imports = (
        "import repercep.attention\nfrom repercep_runtime_b200 import integration\n"
        if order == "reference_first"
        else "from repercep_runtime_b200 import integration\nintegration.install()\nimport repercep.attention\n"
    )
    r = run(
        FAKE_DIFFUSERS
        + FORCE_B200
        + imports,
        """
        import json, torch
        integration.install()
        from diffusers.models.attention_dispatch import (
            AttentionBackendName, _AttentionBackendRegistry, dispatch_attention_fn)
        import repercep.attention.diffusers_backend as ref_bridge
        from repercep.attention.wan_processor import install_repercep_wan_attention
        from repercep_runtime_b200.attention import diffusers_backend as ours
        member = AttentionBackendName("repercep_fp8")
        reg = _AttentionBackendRegistry._backends

        class Transformer:
            processor = None
            def set_attn_processor(self, p):
                self.processor = p

        class Pipe:
            transformer = Transformer()
            transformer_2 = Transformer()

        pipe = Pipe()
        n = install_repercep_wan_attention(pipe)
        wan_fn = reg[pipe.transformer.processor._attention_backend]
        activated = ref_bridge.maybe_activate_from_env()
        calls = []
        prev = ours.handoff_target()
        ours._PREVIOUS["fn"] = lambda *a, **k: calls.append(1) or prev(*a, **k)
        q = torch.randn(1, 64, 2, 32)
        out = dispatch_attention_fn(q, q, q)
        ref = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2), q.transpose(1, 2), q.transpose(1, 2)).transpose(1, 2)
        print(json.dumps({
            "registered": reg[member] is ours._repercep_fp8_attention,
            "previous_is_reference": prev is ref_bridge._repercep_fp8_attention,
            "wan_installed": n, "wan_reaches_b200": wan_fn is ours._repercep_fp8_attention,
            "cosmos_activation": activated and _AttentionBackendRegistry._active_backend == member,
            "ref_bridge_op": type(getattr(ref_bridge._repercep_fp8_attention, "_op", None)).__name__,
            "handed_off": len(calls), "handoff_matches_sdpa": bool(torch.allclose(out, ref, atol=1e-6))}))
        """,
        env_extra={"REPERCEP_FP8_ATTENTION": "1"},
    )
    assert r["registered"] and r["previous_is_reference"], r
    assert r["wan_installed"] == 2 and r["wan_reaches_b200"], r
    assert r["cosmos_activation"], r
    assert r["ref_bridge_op"] == "B200FP8Attention", r
    assert r["handed_off"] == 1 and r["handoff_matches_sdpa"], r


def test_install_without_the_reference_is_a_no_op():
    env = dict(os.environ)
    env["PYTHONPATH"] = str(REPO)
    proc = subprocess.run(
        [sys.executable, "-c",
         "import json; from repercep_runtime_b200 import integration; print(json.dumps(integration.install()))"],
        env=env, capture_output=True, text=True, timeout=120, cwd=str(REPO))
    assert proc.returncode == 0, proc.stderr
    assert "not importable" in json.loads(proc.stdout.strip().splitlines()[-1])["reference"]
