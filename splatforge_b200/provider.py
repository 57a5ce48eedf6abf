"""Registration of the B200 provider behind SplatForge's core runtime and renderer registry.

Operator seam (src/splatforge/gaussian/ops.py:175-254, src/splatforge/core/models.py:112-172):
``implementations()`` returns ``SimpleNamespace(manifest, runner, support)`` objects and
``capabilities()`` their ``CapabilityRecord``s, in the shape
``create_surface_runtime(implementations=..., capabilities=...)`` consumes, exactly as the
reference's own CUDA composite provider does (providers/torch/gaussian/cuda_composite.py:90-136).
Every manifest names provider ``native_cuda`` (the first provider of the default
``ExecutionPolicy``), devices ``["cuda"]``, dtype ``float32`` and the sha256 of the installed
``semantics.json`` as its ``op_spec_revision``.  The culled opacity field is registered as a
second implementation of ``gaussian.opacity_field@1`` that declares host synchronisation
(one candidate-count read per origin); the default policy (``host_sync="forbid"``) refuses
it, so it runs only when selected explicitly under a policy that allows it.

Renderer seam (src/splatforge/studio/renderers.py:356-439): ``register_renderer(renderers)``
adds the ``b200`` backend; the same factory is published as the ``splatforge.renderers``
entry point ``b200`` in pyproject.toml.
"""

from __future__ import annotations

import hashlib
from importlib.resources import files
from pathlib import Path
from types import SimpleNamespace

from . import ops
from .renderer import b200_factory

PROVIDER = "native_cuda"
VERSION = "0.1.0"
CSRC = Path(__file__).resolve().parent / "csrc"

# op key -> (implementation id, runner, lowering target, variant, backward, sources)
_OPS = {
    "gaussian.covariance@1": ("splatforge_b200.native_cuda.covariance.v1", ops.covariance, "sf_b200_covariance_forward",
                              "sm100a-float32", True, ("preprocess.cu", "sf_math.cuh", "sf_grad.cuh")),
    "gaussian.sh_color@1": ("splatforge_b200.native_cuda.sh_color.v1", ops.sh_color, "sf_b200_sh_color_forward",
                            "sm100a-float32", True, ("preprocess.cu", "sf_math.cuh")),
    "splat.alpha_composite@3": ("splatforge_b200.native_cuda.alpha_composite.v3", ops.alpha_composite_selected,
                                "sf_b200_alpha_composite_forward", "sm100a-float32-selected", True,
                                ("composite.cu", "sf_device.cuh")),
    "splat.alpha_composite@2": ("splatforge_b200.native_cuda.alpha_composite.v2", ops.alpha_composite_batch,
                                "sf_b200_alpha_composite_forward", "sm100a-float32-batched", True,
                                ("composite.cu", "sf_device.cuh")),
    "splat.alpha_composite@1": ("splatforge_b200.native_cuda.alpha_composite.v1", ops.alpha_composite,
                                "sf_b200_alpha_composite_forward", "sm100a-float32", True,
                                ("composite.cu", "sf_device.cuh")),
    "gaussian.opacity_field@1": ("splatforge_b200.native_cuda.opacity_field.v1", ops.opacity_field,
                                 "sf_b200_opacity_field", "sm100a-float32-forward", False, ("opacity_field.cu",)),
    "camera.pixel_rays@1": ("splatforge_b200.native_cuda.pixel_rays.v1", ops.pixel_rays, "sf_b200_pixel_rays",
                            "sm100a-float32-forward", False, ("geometry.cu",)),
    "gaussian.ray_peak@1": ("splatforge_b200.native_cuda.ray_peak.v1", ops.ray_peak, "sf_b200_ray_peak",
                            "sm100a-float32-forward", False, ("geometry.cu",)),
    "geometry.depth_normals@1": ("splatforge_b200.native_cuda.depth_normals.v1", ops.depth_normals,
                                 "sf_b200_depth_normals", "sm100a-float32", True, ("geometry.cu",)),
    "matching.patch_zncc@1": ("splatforge_b200.native_cuda.patch_zncc.v1", ops.patch_zncc, "sf_b200_patch_zncc",
                              "sm100a-float32", True, ("training.cu", "sf_device.cuh")),
    "gaussian.sh_ambiguity@1": ("splatforge_b200.native_cuda.sh_ambiguity.v1", ops.sh_ambiguity,
                                "sf_b200_sh_ambiguity", "sm100a-float32", True, ("training.cu", "sf_device.cuh")),
    "gaussian.ray_color_variance@1": ("splatforge_b200.native_cuda.ray_color_variance.v1", ops.ray_color_variance,
                                      "sf_b200_ray_color_variance", "sm100a-float32", True,
                                      ("composite.cu", "sf_device.cuh")),
    "gaussian.ray_color_variance@2": ("splatforge_b200.native_cuda.ray_color_variance.v2",
                                      ops.ray_color_variance_batch, "sf_b200_ray_color_variance",
                                      "sm100a-float32-batched", True, ("composite.cu", "sf_device.cuh")),
}

# Additional implementations of an operator already listed above, selected explicitly
# (not by selection()): the culled opacity field synchronises the host once per origin,
# so only a policy that allows declared host synchronisation may run it.
_ALTERNATIVES = {
    "splatforge_b200.native_cuda.opacity_field_culled.v1": (
        "gaussian.opacity_field@1", ops.opacity_field_culled, "sf_b200_opacity_field_culled",
        "sm100a-float32-forward-culled", False, ("opacity_field.cu", "binning.cu"), "per_origin"),
}


def spec_revision():
    """sha256 of the installed SplatForge semantics.json (its operators' revision)."""
    contents = files("splatforge.gaussian").joinpath("semantics.json").read_bytes()
    return "sha256:" + hashlib.sha256(contents).hexdigest()


def build_fingerprint(sources):
    h = hashlib.sha256()
    for name in sources:
        h.update((CSRC / name).read_bytes())
    return "sha256:" + h.hexdigest()


def _entry(key):
    """(op, implementation id, runner, target, variant, backward, sources, host sync) of an
    operator key (its default implementation) or of an alternative implementation id."""
    if key in _OPS:
        identifier, runner, target, variant, backward, sources = _OPS[key]
        return key, identifier, runner, target, variant, backward, sources, "none"
    op, runner, target, variant, backward, sources, sync = _ALTERNATIVES[key]
    return op, key, runner, target, variant, backward, sources, sync


def manifest_dict(key, revision):
    op, identifier, runner, target, variant, backward, sources, sync = _entry(key)
    return {
        "schema_version": 1,
        "implementation_id": identifier,
        "provider": PROVIDER,
        "provider_api": 1,
        "op": op,
        "op_spec_revision": revision,
        "implementation_version": VERSION,
        "lowering_target": f"libsf_b200.{target}",
        "static_variant_token": variant,
        "priority": 0,
        "declared_eligibility": {
            "devices": ["cuda"],
            "dtypes": ["float32"],
            "layouts": ["contiguous", "strided_last_dim", "strided"],
            "backward": backward,
            "jvp": False,
            "determinism_guarantee": "none",
            "host_synchronization": sync,
            "cuda_graph": False,
            "execution": {"eager": "supported"},
        },
        "build": {"fingerprint": build_fingerprint(sources)},
    }


def _keys(ops_keys):
    """Default implementations of the given operators (all by default), followed by the
    alternatives of those operators."""
    ops_list = list(ops_keys or _OPS)
    return ops_list + [alt for alt, entry in _ALTERNATIVES.items() if entry[0] in ops_list]


def implementations(ops_keys=None):
    """Manifests + runners for SplatForge's ``create_surface_runtime``: every operator's
    default implementation plus the alternatives (selected only by explicit id)."""
    from splatforge.core.models import ImplementationManifest

    revision = spec_revision()
    out = []
    for key in _keys(ops_keys):
        manifest = ImplementationManifest.from_dict(manifest_dict(key, revision))
        out.append(SimpleNamespace(manifest=manifest, runner=_entry(key)[2], support=None))
    return out


def capabilities(ops_keys=None):
    from splatforge.core.models import CapabilityRecord

    return [
        CapabilityRecord(_entry(key)[1], "experimental", "splatforge-b200", "b200-sm100a")
        for key in _keys(ops_keys)
    ]


def selection(ops_keys=None, *, culled_field=False):
    """``{op: implementation_id}`` for ``SurfaceOperators(runtime, implementations=...)``.
    ``culled_field`` selects the culled opacity field, which needs an execution policy
    with ``host_sync="allow_declared"``."""
    sel = {op: _OPS[op][0] for op in ops_keys or _OPS}
    if culled_field and "gaussian.opacity_field@1" in sel:
        sel["gaussian.opacity_field@1"] = "splatforge_b200.native_cuda.opacity_field_culled.v1"
    return sel


def surface_operators(ops_keys=None):
    """A sealed runtime with the B200 implementations registered, and the
    ``SurfaceOperators`` facade selecting them by exact id."""
    from splatforge.gaussian import SurfaceOperators
    from splatforge.gaussian.ops import create_surface_runtime

    runtime = create_surface_runtime(implementations=implementations(ops_keys), capabilities=capabilities(ops_keys))
    return SurfaceOperators(runtime, implementations=selection(ops_keys))


def register_renderer(registry=None, name="b200"):
    """Add the B200 backend to a ``ComponentRegistry`` (default: Studio's ``renderers``)."""
    if registry is None:
        from splatforge.studio.renderers import renderers as registry
    registry.register(name, b200_factory)
    return registry


def register_exporter(registry=None, name="b200-gof"):
    """Add the device GOF exporter to a ``ComponentRegistry`` (default: Studio's
    ``exporters``, src/splatforge/studio/exporters.py:264-266)."""
    if registry is None:
        from splatforge.studio.exporters import exporters as registry
    from .meshing import B200GOFExporter

    registry.register(name, B200GOFExporter)
    return registry
