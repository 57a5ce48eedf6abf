"""Registration behind SplatForge's own core runtime and renderer registry (CPU).

Uses the reference package where it is importable (``SPLATFORGE_SRC`` pointing at its
``src`` directory, or the baseline/_ref install; it is not shipped with this
repository); skipped otherwise.  No device is needed: dispatch is metadata-only
(src/splatforge/core/runtime.py:256-326).
"""

from __future__ import annotations

import sys

import pytest
import torch

from tests._util import reference_source

REF = reference_source()
if REF is None:
    pytest.skip("the SplatForge reference package is not importable", allow_module_level=True)
sys.path.insert(0, str(REF))
sys.dont_write_bytecode = True

from splatforge.core.errors import DispatchError  # noqa: E402
from splatforge.core.policy import ExecutionPolicy  # noqa: E402
from splatforge.gaussian.ops import create_surface_runtime  # noqa: E402
from splatforge.studio.plugins import ComponentRegistry  # noqa: E402

from splatforge_b200 import provider  # noqa: E402
from splatforge_b200.renderer import B200Renderer  # noqa: E402


def test_manifests_register_with_the_current_spec_revision():
    runtime = create_surface_runtime(implementations=provider.implementations(), capabilities=provider.capabilities())
    for op, identifier in provider.selection().items():
        impl = runtime.implementations.get(identifier)
        assert impl is not None and str(impl.manifest.op_key) == op
        assert impl.manifest.provider == "native_cuda"
        assert impl.manifest.eligibility.devices == ("cuda",)
        assert impl.manifest.op_spec_revision == provider.spec_revision()


def test_native_provider_is_first_in_the_default_policy_order_for_cuda_inputs():
    runtime = create_surface_runtime(implementations=provider.implementations(), capabilities=provider.capabilities())
    q = torch.randn(4, 4, device="meta")
    s = torch.rand(4, 3, device="meta")
    # metadata-only explanation with an unverified-allowed exact selection
    policy = ExecutionPolicy(implementation_id=provider.selection()["gaussian.covariance@1"], allow_unverified=True)
    exp = runtime.explain_dispatch("gaussian.covariance@1", q, s, policy=policy)
    cand = [c for c in exp.candidates if c.implementation_id == policy.implementation_id][0]
    assert "unsupported_device" in cand.reasons  # meta is not cuda: no silent acceptance


def test_no_fallback_for_cpu_tensors():
    ops = provider.surface_operators()
    q = torch.randn(4, 4)
    s = torch.rand(4, 3)
    with pytest.raises(DispatchError):
        ops("gaussian.covariance@1", q, s)


def test_opacity_field_declares_no_backward():
    runtime = create_surface_runtime(implementations=provider.implementations(), capabilities=provider.capabilities())
    impl = runtime.implementations.get(provider.selection()["gaussian.opacity_field@1"])
    assert impl.manifest.eligibility.backward is False


def test_renderer_factory_registers_and_builds():
    reg = ComponentRegistry("splatforge.renderers.test")
    provider.register_renderer(reg)
    from splatforge.studio.config import RenderConfig

    r = reg.get("b200")(RenderConfig(), mode="gof", trunc_sigma=2.0, ops=None)
    assert isinstance(r, B200Renderer)
    with pytest.raises(ValueError):
        reg.register("b200", object())  # duplicate names raise (plugins.py:14-18)
    # render_training keeps the per-mode distortion profile (batched_renderer.py:37-43)
    calls = []
    r.render = lambda scene, camera, selected=None, distortions="both": calls.append(distortions)
    r.render_training(None, None, geometric=True)
    r.mode = "radegs"
    r.render_training(None, None, geometric=True)
    r.mode = "ambisur"
    r.render_training(None, None, geometric=True)
    r.mode = "gof"
    r.render_training(None, None, geometric=False)
    assert calls == ["l1", "l2", "none", "none"]


def test_geometry_ops_and_the_culled_field_register():
    runtime = create_surface_runtime(implementations=provider.implementations(), capabilities=provider.capabilities())
    sel = provider.selection()
    for op in ("camera.pixel_rays@1", "gaussian.ray_peak@1", "geometry.depth_normals@1", "matching.patch_zncc@1",
               "gaussian.sh_ambiguity@1", "gaussian.ray_color_variance@1", "gaussian.ray_color_variance@2",
               "splat.alpha_composite@1", "splat.alpha_composite@2"):
        impl = runtime.implementations.get(sel[op])
        assert impl is not None and str(impl.manifest.op_key) == op
    assert runtime.implementations.get(sel["geometry.depth_normals@1"]).manifest.eligibility.backward is True
    culled = provider.selection(culled_field=True)["gaussian.opacity_field@1"]
    impl = runtime.implementations.get(culled)
    assert str(impl.manifest.op_key) == "gaussian.opacity_field@1"
    assert impl.manifest.eligibility.host_synchronization != "none"
    # the default policy forbids host synchronisation: the culled field is refused
    p = torch.randn(5, 3, device="meta")
    policy = ExecutionPolicy(implementation_id=culled, allow_unverified=True)
    exp = runtime.explain_dispatch("gaussian.opacity_field@1", p, torch.randn(4, 3, device="meta"),
                                   torch.randn(4, 3, 3, device="meta"), torch.rand(4, device="meta"),
                                   torch.randn(2, 3, device="meta"), policy=policy)
    cand = [c for c in exp.candidates if c.implementation_id == culled][0]
    assert "host_synchronization_forbidden" in cand.reasons
    # a policy that allows declared host synchronisation clears that reason
    allowed = ExecutionPolicy(implementation_id=culled, providers=("native_cuda",), allow_unverified=True,
                              host_sync="allow_declared")
    exp = runtime.explain_dispatch("gaussian.opacity_field@1", p, torch.randn(4, 3, device="meta"),
                                   torch.randn(4, 3, 3, device="meta"), torch.rand(4, device="meta"),
                                   torch.randn(2, 3, device="meta"), policy=allowed)
    cand = [c for c in exp.candidates if c.implementation_id == culled][0]
    assert "host_synchronization_forbidden" not in cand.reasons


def test_device_gof_exporter_registers():
    """``b200-gof`` joins an exporter registry beside the reference's ``gof``
    (exporters.py:264-266) and exposes the same ``export(pipeline, path, config)`` call."""
    from splatforge.studio.exporters import GOFExporter

    from splatforge_b200.meshing import B200GOFExporter

    reg = ComponentRegistry("splatforge.exporters.test")
    reg.register("gof", GOFExporter)
    provider.register_exporter(reg)
    assert reg.get("b200-gof") is B200GOFExporter
    assert callable(reg.get("b200-gof")().export)
    with pytest.raises(ValueError):
        provider.register_exporter(reg)  # duplicate names raise (plugins.py:14-18)
