"""Communication engines (NVLink kernels, torch over a transport) and the symmetric heap."""
