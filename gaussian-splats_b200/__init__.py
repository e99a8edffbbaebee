"""B200-native Gaussian-splat rasterizer.

Drop-in for the reference's ``gaussian_splats::rasterize`` operator and its
``splats`` API: projection, tile binning and per-tile compositing, forward and
backward, as hand-written sm_100a CUDA kernels behind a C-ABI library
(``libgs_b200.so``, declared in ``include/gs_b200.h``).

Submodules are imported on demand so that the host-only parts (cameras,
scenes, checkpoints) work without the native library; the rasterizer itself
raises if the library is missing.
"""

__version__ = "0.1.0"
