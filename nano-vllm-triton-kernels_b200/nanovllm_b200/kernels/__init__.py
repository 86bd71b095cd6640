# The B200 kernel package, laid out as the reference's nanovllm/kernels (__init__.py, qk_norm_rope_kv.py,
# rms_norm.py, swiglu.py, matmul.py). `backend` names this implementation: nano-vllm selects kernels by the
# string in nanovllm.kernels.backend (nanovllm/kernels/__init__.py:1-5); nanovllm_b200.install() sets it to "b200".
backend = "b200"
