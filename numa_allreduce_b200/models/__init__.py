"""Model families built on the fused tensor-parallel ops."""
