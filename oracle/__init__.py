"""CPU oracle for the CCQ cleaning operator: test infrastructure, never the product path."""
