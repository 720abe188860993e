"""Test-only oracle of the LUMA step (see luma_ref.py).  Not part of the product."""
