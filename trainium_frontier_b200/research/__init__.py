"""Research tooling around the trainer: checkpoint averaging, evaluation reconciliation,
an experiment runner that logs each run's summary, and the short single-GPU
autoresearch loop."""
