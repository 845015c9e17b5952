"""CPU oracle of the indexer (test infrastructure only; see oracle/oracle.py)."""
