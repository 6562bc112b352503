"""orchestration"""
