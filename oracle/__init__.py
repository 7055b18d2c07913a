"""CPU oracle for the quantized Llama-layer path.

TEST INFRASTRUCTURE ONLY. Nothing in the ``orchard_b200`` product imports,
links or executes this package. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference legs may use it, and only as the
checker or as the timed CPU stand-in for the reference implementation.

Parity pin: the quantizer restatement is checked bit-exactly against outputs of
the reference's own ``orchard/quantizer.py`` (fixtures in ``tests/golden/``),
and the layer / generate restatement against outputs of the reference's own
``orchard/model.py`` run on CPU through a literal transcription of the Metal
kernels (``tests/golden/make_golden.py``).
"""

from . import ops  # noqa: F401
from . import model  # noqa: F401
