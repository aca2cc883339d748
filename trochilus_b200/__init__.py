"""trochilus_b200: the OLMoE MoE-layer hot path of Trochilus on the B200. The product is the C library libtrmoe.so
(csrc/, built by build.py, declared in include/trmoe.h); moe.py binds it for Python, ep.py drives expert parallelism
across GPUs, gguf_blocks.py writes synthetic GGUF blocks, timeline.py reads the decode kernel's trace."""
