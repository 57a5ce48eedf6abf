"""CPU oracle for the Gaussian-splatting hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch (CPU, float32/float64) and numpy, the
algorithm of SplatForge's Torch provider for the rasterizer path:

* ``oracle.ops``      -- ``gaussian.covariance@1``, ``gaussian.sh_color@1``,
                         ``camera.pixel_rays@1``, ``gaussian.ray_peak@1``,
                         ``splat.alpha_composite@1/@2/@3``,
                         ``gaussian.ray_color_variance@1/@2``,
                         ``gaussian.opacity_field@1``
                         (src/splatforge/providers/torch/gaussian/reference.py)
* ``oracle.binning``  -- exact tile lists in stable depth order
                         (src/splatforge/studio/tile_binning.py:10-34)
* ``oracle.render``   -- the tiled renderer with its three rendering modes
                         (src/splatforge/studio/renderers.py:76-353,
                         src/splatforge/studio/batched_renderer.py:37-410)

Parity of this oracle is pinned by ``tests/test_oracle_golden.py`` against
fixtures under ``tests/golden/`` that ``tests/golden/make_golden.py`` produced
by running the reference itself.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline
leg and ``--impl reference``) may import this package, and only as the checker
or the timed CPU baseline.  The product package ``splatforge_b200`` never
imports it and has no CPU fallback.
"""
