! Drop-in replacement of module matmul_3p5bit_groq (matmul_3p5bit_dynamic.f90) over
! libq35.so: same module name, procedure names, argument order and intents.
! Link: gfortran -c matmul_3p5bit_groq.f90 && ... -L<pkg> -lq35 -Wl,-rpath,<pkg>
module matmul_3p5bit_groq
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float
    use iso_fortran_env, only: int8, int32, real32
    implicit none
    private
    public :: matmul_3p5bit_awq, dequantize_output_3p5bit

    interface
        ! the reference procedure is already bind(C) with value M, N, K
        subroutine matmul_3p5bit_awq(A, W_Q, W_scales, W_offsets, C, M, N, K) &
                bind(C, name="matmul_3p5bit_awq")
            import :: c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(M, K)
            integer(c_int8_t), intent(in) :: W_Q(K/2, N)
            real(c_float), intent(in) :: W_scales(N), W_offsets(N)
            integer(c_int32_t), intent(out) :: C(M, N)
        end subroutine matmul_3p5bit_awq

        integer(c_int) function q35_dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N) &
                bind(C, name="q35_dequantize_output_3p5bit")
            import :: c_int, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N
            integer(c_int32_t), intent(in) :: C(M, N)
            real(c_float), intent(in) :: W_scales(N), W_offsets(N)
            real(c_float), intent(out) :: Out(M, N)
        end function q35_dequantize_output_3p5bit
    end interface

contains

    ! matmul_3p5bit_dynamic.f90:69-82
    subroutine dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N)
        integer(int32), intent(in), value :: M, N
        integer(int32), intent(in) :: C(M, N)
        real(real32), intent(in) :: W_scales(N), W_offsets(N)
        real(real32), intent(out) :: Out(M, N)
        if (q35_dequantize_output_3p5bit(C, W_scales, W_offsets, Out, M, N) /= 0) &
            error stop "dequantize_output_3p5bit: libq35 failed"
    end subroutine dequantize_output_3p5bit

end module matmul_3p5bit_groq
