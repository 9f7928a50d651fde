"""Parity oracle for treeattn_b200 (test infrastructure only; never a product code path)."""
