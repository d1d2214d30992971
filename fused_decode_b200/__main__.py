"""``python -m fused_decode_b200`` runs the per-operator results table, as
``python -m fused_decode`` does in the reference (src/fused_decode/__main__.py)."""

from fused_decode_b200.bench import main

if __name__ == "__main__":
    main()
