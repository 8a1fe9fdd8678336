"""logging"""
