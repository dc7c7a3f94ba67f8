"""Multi-GPU (Ulysses SP) leg of bench.py."""


def run_sequence_parallel(args):
    raise NotImplementedError("Ulysses SP bench leg is not built yet")
