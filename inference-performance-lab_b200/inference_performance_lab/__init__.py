"""B200-native (sm_100a) fused add+RMSNorm and SiLU-and-mul ops.

Same import paths as the reference package: ``inference_performance_lab.kernels.extension``
holds the op wrappers, ``inference_performance_lab.kernels.vllm_plugin`` the vLLM IR provider.
The kernels live in the in-tree ``_native/`` libraries built by ``build.py``.
"""
