"""tfimage on B200: the quantized-linear hot path of the Qwen-Image DiT engine (linear, kernels, ext) rebuilt on
hand-written sm_100a kernels in libtfb.so. The DiT, calibration and ComfyUI node of the reference import
``tfimage.linear`` / ``tfimage.kernels`` and run on top of it unchanged."""

__version__ = "0.1.0"
