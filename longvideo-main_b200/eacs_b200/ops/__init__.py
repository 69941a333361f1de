"""Operator modules mirroring cst_ssm/ops (same names and argument meaning)."""
