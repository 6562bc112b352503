"""router"""
