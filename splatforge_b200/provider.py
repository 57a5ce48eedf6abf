"""Registration of the B200 provider behind SplatForge's core runtime and renderer registry.

Operator seam (src/splatforge/gaussian/ops.py:175-254, src/splatforge/core/models.py:112-172):
``implementations()`` returns ``SimpleNamespace(manifest, runner, support)`` objects and
``capabilities()`` their ``CapabilityRecord``s, in the shape
``create_surface_runtime(implementations=..., capabilities=...)`` consumes, exactly as the
reference's own CUDA composite provider does (providers/torch/gaussian/cuda_composite.py:90-136).
Every manifest names provider ``native_cuda`` (the first provider of the default
``ExecutionPolicy``), devices ``["cuda"]``, dtype ``float32`` and the sha256 of the installed
``semantics.json`` as its ``op_spec_revision``.

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
    "gaussian.opacity_field@1": ("splatforge_b200.native_cuda.opacity_field.v1", ops.opacity_field,
                                 "sf_b200_opacity_field", "sm100a-float32-forward", False, ("opacity_field.cu",)),
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


def manifest_dict(op, revision):
    identifier, runner, target, variant, backward, sources = _OPS[op]
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
            "host_synchronization": "none",
            "cuda_graph": False,
            "execution": {"eager": "supported"},
        },
        "build": {"fingerprint": build_fingerprint(sources)},
    }


def implementations(ops_keys=None):
    """Manifests + runners for SplatForge's ``create_surface_runtime``."""
    from splatforge.core.models import ImplementationManifest

    revision = spec_revision()
    out = []
    for op in ops_keys or _OPS:
        manifest = ImplementationManifest.from_dict(manifest_dict(op, revision))
        out.append(SimpleNamespace(manifest=manifest, runner=_OPS[op][1], support=None))
    return out


def capabilities(ops_keys=None):
    from splatforge.core.models import CapabilityRecord

    return [
        CapabilityRecord(_OPS[op][0], "experimental", "splatforge-b200", "b200-sm100a")
        for op in ops_keys or _OPS
    ]


def selection(ops_keys=None):
    """``{op: implementation_id}`` for ``SurfaceOperators(runtime, implementations=...)``."""
    return {op: _OPS[op][0] for op in ops_keys or _OPS}


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
