"""The B200 kernel modules, laid out as the reference's nanovllm/kernels package (qk_norm_rope_kv.py, rms_norm.py,
swiglu.py, matmul.py) plus attention.py for the attention layer's KV-cache write and decode attention. The reference
picks its kernels by the string nanovllm.kernels.backend (nanovllm/kernels/__init__.py:1-5); nanovllm_b200.install()
adds "b200" to that switch."""
