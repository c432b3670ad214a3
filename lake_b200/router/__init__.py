"""Request router: HTTP front, node pick, execution-mode selection, priority
admission and the view/load/autoscale loops (C++ cores in lake_b200._host)."""
