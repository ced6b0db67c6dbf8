"""CPU oracle of the FOLD path (test infrastructure; never imported by the product package)."""
