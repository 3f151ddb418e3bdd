"""The engine-module contract of FoldForge's Pairformer pair stack, with the ``b200`` backend."""
