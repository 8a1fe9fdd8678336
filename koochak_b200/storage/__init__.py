"""Persistence: write-once stores, checkpoint publication, collections and transfer."""

__all__: list = []
