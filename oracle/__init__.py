"""CPU oracle for the DIP decode path: test infrastructure, never imported by
the product.  See dip_oracle.py."""
