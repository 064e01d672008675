"""NVFP4 test oracle (TEST INFRASTRUCTURE ONLY; never imported by the product)."""
