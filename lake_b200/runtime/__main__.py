"""`python -m lake_b200.runtime` starts one worker (role and model from LAKE_* env vars)."""
from .worker import main

main()
