"""mod_b200: a Blackwell (B200, sm_100a) native LLM/VLM inference engine.

Public entry points:
  * :class:`mod_b200.engine.llm_engine.LLMEngine` - continuous-batching engine
  * :mod:`mod_b200.api` - model plugins (Inference-PIO style plugin API)
  * :mod:`mod_b200.config` - model / runtime configuration
"""
__version__ = "0.1.0"
