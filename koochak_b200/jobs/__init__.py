"""jobs"""
