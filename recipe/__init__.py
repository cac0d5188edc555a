"""Recipes: declarative run definitions (``SERVICE_GROUPS``, ``COLOCATIONS``, ``main()``)."""
