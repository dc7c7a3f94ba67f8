"""Seeded synthetic inputs for the benchmark configurations (test infrastructure).

The generators live in ``eraserdit_b200.synthetic`` so that the benchmark can
draw the same inputs without importing this package; they are re-exported
here for the tests and the golden-vector script.
"""

from eraserdit_b200.synthetic import (  # noqa: F401
    CONFIG0, CONFIG1, LayerConfig, LayerWeights, make_hidden, make_params)
