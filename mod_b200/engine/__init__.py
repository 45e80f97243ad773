from .sequence import SamplingParams, Sequence, SeqStatus  # noqa: F401
