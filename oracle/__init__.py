"""CPU oracle (test infrastructure): a numpy restatement of willow's MoE path, used only by tests/, smoke() and
bench.py's CPU-baseline leg as the checker. Never imported by the product package."""
