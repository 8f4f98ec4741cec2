"""Model-level building blocks on top of the communication buffer."""
