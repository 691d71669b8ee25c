"""Model families beyond the transformer stack, one module per reference model crate:
``rnn`` (brain-rnn), ``cv`` (brain-cv), ``gnn`` (brain-gnn), ``diffusion`` (brain-diffusion),
``gan`` (brain-gan), ``rl`` (brain-rl), ``audio`` (brain-audio), ``neuroevolution``
(brain-neuroevolution). Transformers and ViT live in ``brain_b200.models``."""
from . import audio, cv, diffusion, gan, gnn, neuroevolution, rl, rnn  # noqa: F401
