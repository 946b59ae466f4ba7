"""Device operators: thin kernel wrappers (``kernels``), autograd functions of the
fused GPT path (``fused``), attention and FP8 quantisation."""
