"""ElasticMegatron-B200: an elastic LLM training framework for NVIDIA B200."""
__version__ = "0.1.0"
