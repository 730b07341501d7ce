"""CPU restatement of the reference path (test infrastructure: the checker, never the product)."""
