"""`python -m lake_b200.router` starts the HTTP router (LAKE_* env vars)."""
from .http import main

main()
