"""gRPC services of the pool and the node: ControlPlaneService over the C++
authority, AgentService, TransferService and TcpDataService over the C++
transfer engine and byte store."""
